// denoiser::Conv2dLayer — source-compatible with the reference's
// include/denoiser/layers/conv2d.h:33-100, over dn_conv2d_* (one
// implicit-GEMM tensor-core kernel per call, bias fused).
#pragma once

#include <optional>
#include <stdexcept>
#include <string>

#include "denoiser/detail/abi.h"
#include "denoiser/tensor.h"
#include "denoiser/weight_loader.h"
#include "denoiser_b200_layers.h"

namespace denoiser {

class Conv2dLayer {
public:
    Conv2dLayer(const WeightStore& store, const std::string& weight_name,
                std::optional<std::string> bias_name = std::nullopt, int pad = 1, int stride = 1, int dilation = 1,
                int groups = 1) {
        int dev = 0;
        CUDA_CHECK(cudaGetDevice(&dev));
        detail::check(dn_conv2d_create(store.handle(), weight_name.c_str(), bias_name ? bias_name->c_str() : nullptr,
                                       pad, stride, dilation, groups, dev, &h_));
        detail::check(dn_conv2d_info(h_, &out_channels_, &in_channels_, &kernel_h_, &kernel_w_, &groups_));
    }
    ~Conv2dLayer() { dn_conv2d_destroy(h_); }
    Conv2dLayer(const Conv2dLayer&) = delete;
    Conv2dLayer& operator=(const Conv2dLayer&) = delete;

    // FP16 NCHW in, newly allocated FP16 NCHW out (conv2d.cu:94-150).
    Tensor forward(const Tensor& input, cudaStream_t stream = nullptr) const {
        if (input.dtype() != DType::kFloat16) throw std::runtime_error("Conv2dLayer::forward: expected FP16 input");
        int ho = 0, wo = 0;
        detail::check(dn_conv2d_output_size(h_, static_cast<int>(input.height()), static_cast<int>(input.width()), &ho, &wo));
        Tensor out = Tensor::empty({input.batch(), out_channels_, ho, wo}, DType::kFloat16);
        detail::check(dn_conv2d_forward(h_, input.data(), static_cast<int>(input.batch()), static_cast<int>(input.channels()),
                                        static_cast<int>(input.height()), static_cast<int>(input.width()), out.data(), stream));
        return out;
    }

    int out_channels() const noexcept { return out_channels_; }
    int in_channels() const noexcept { return in_channels_; }
    int kernel_h() const noexcept { return kernel_h_; }
    int kernel_w() const noexcept { return kernel_w_; }
    int groups() const noexcept { return groups_; }

private:
    dn_conv2d* h_ = nullptr;
    int out_channels_ = 0, in_channels_ = 0, kernel_h_ = 0, kernel_w_ = 0, groups_ = 1;
};

}  // namespace denoiser
