// denoiser::DeformConv2dLayer — source-compatible with the reference's
// include/denoiser/layers/deform_conv2d.h:11-55, over dn_dcn_* (one fused
// sampling + tensor-core kernel per call; no im2col buffer, no cuBLAS).
#pragma once

#include <stdexcept>
#include <string>

#include "denoiser/detail/abi.h"
#include "denoiser/tensor.h"
#include "denoiser/weight_loader.h"
#include "denoiser_b200_layers.h"

namespace denoiser {

class DeformConv2dLayer {
public:
    DeformConv2dLayer(const WeightStore& store, const std::string& weight_name, const std::string& bias_name,
                      int pad = 1, int stride = 1, int dilation = 1, int deform_groups = 8) {
        int dev = 0;
        CUDA_CHECK(cudaGetDevice(&dev));
        detail::check(dn_dcn_create(store.handle(), weight_name.c_str(), bias_name.c_str(), pad, stride, dilation,
                                    deform_groups, dev, &h_));
        int kh = 0, kw = 0;
        detail::check(dn_dcn_info(h_, &out_channels_, &in_channels_, &deform_groups_, &kh, &kw));
    }
    ~DeformConv2dLayer() { dn_dcn_destroy(h_); }
    DeformConv2dLayer(const DeformConv2dLayer&) = delete;
    DeformConv2dLayer& operator=(const DeformConv2dLayer&) = delete;

    Tensor forward(const Tensor& input, const Tensor& offsets, const Tensor& masks, cudaStream_t stream = nullptr) const {
        if (input.dtype() != DType::kFloat16 || offsets.dtype() != DType::kFloat16 || masks.dtype() != DType::kFloat16)
            throw std::runtime_error("DeformConv2dLayer::forward: all inputs must be FP16");
        int ho = 0, wo = 0;
        detail::check(dn_dcn_output_size(h_, static_cast<int>(input.height()), static_cast<int>(input.width()), &ho, &wo));
        Tensor out = Tensor::empty({input.batch(), out_channels_, ho, wo}, DType::kFloat16);
        detail::check(dn_dcn_forward(h_, input.data(), offsets.data(), masks.data(), static_cast<int>(input.batch()),
                                     static_cast<int>(input.height()), static_cast<int>(input.width()), out.data(), stream));
        return out;
    }

    int out_channels() const noexcept { return out_channels_; }
    int in_channels() const noexcept { return in_channels_; }
    int deform_groups() const noexcept { return deform_groups_; }

private:
    dn_dcn* h_ = nullptr;
    int out_channels_ = 0, in_channels_ = 0, deform_groups_ = 0;
};

}  // namespace denoiser
