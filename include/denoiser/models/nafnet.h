// denoiser::NAFNet — source-compatible with the reference's
// include/denoiser/models/nafnet.h:11-28, over dn_model_* (the B200 engine:
// weights packed once, fused tensor-core kernels, one activation arena).
#pragma once

#include <stdexcept>
#include <vector>

#include "denoiser/detail/abi.h"
#include "denoiser/tensor.h"
#include "denoiser/weight_loader.h"
#include "denoiser_b200.h"

namespace denoiser {

namespace detail {

// One engine instance on the current device, built from the store's manifest.
class EngineHandle {
public:
    explicit EngineHandle(const WeightStore& store) {
        int dev = 0;
        CUDA_CHECK(cudaGetDevice(&dev));
        check(dn_model_create(store.manifest_path().c_str(), dev, &m_));
        check(dn_model_get_info(m_, &info_));
        for (int i = 0; i < info_.num_levels && i < 8; ++i) enc_.push_back(info_.enc_channels[i]);
    }
    ~EngineHandle() { dn_model_destroy(m_); }
    EngineHandle(const EngineHandle&) = delete;
    EngineHandle& operator=(const EngineHandle&) = delete;

    // y (N, 3, H, W) for x of `ndim` dims (4: frames, 5: clips).
    Tensor run(const Tensor& x, int ndim, cudaStream_t stream) const {
        if (x.dtype() != DType::kFloat16) throw std::runtime_error("NAFNet::forward: expected FP16 input");
        const auto& s = x.shape();
        if (static_cast<int>(s.size()) != ndim) throw std::invalid_argument("forward: unexpected input rank");
        // Stream-ordered output: no device-wide synchronisation per frame.
        Tensor y = Tensor::empty({s[0], 3, s[ndim - 2], s[ndim - 1]}, DType::kFloat16, stream);
        check(dn_model_forward(m_, x.data(), s.data(), ndim, y.data(), stream));
        return y;
    }

    const dn_model_info& info() const noexcept { return info_; }
    const std::vector<int>& enc() const noexcept { return enc_; }
    dn_model* handle() const noexcept { return m_; }

private:
    dn_model* m_ = nullptr;
    dn_model_info info_{};
    std::vector<int> enc_;
};

}  // namespace detail

class NAFNet {
public:
    explicit NAFNet(const WeightStore& store) : e_(store) {
        if (e_.info().kind != 0) throw std::runtime_error("NAFNet: the manifest holds a temporal model");
    }
    NAFNet(const NAFNet&) = delete;
    NAFNet& operator=(const NAFNet&) = delete;

    // input (N, C, H, W) FP16 -> denoised (N, 3, H, W) FP16, newly allocated.
    Tensor forward(const Tensor& input, cudaStream_t stream = nullptr) const { return e_.run(input, 4, stream); }

    const std::vector<int>& enc_channels() const noexcept { return e_.enc(); }
    int num_levels() const noexcept { return e_.info().num_levels; }
    int in_channels() const noexcept { return e_.info().in_channels; }

private:
    detail::EngineHandle e_;
};

}  // namespace denoiser
