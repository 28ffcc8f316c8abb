// denoiser::UpsampleLayer — source-compatible with the reference's
// include/denoiser/layers/upsample.h:17-38, over dn_upsample_bilinear.
#pragma once

#include <stdexcept>

#include "denoiser/detail/abi.h"
#include "denoiser/tensor.h"
#include "denoiser_b200_ops.h"

namespace denoiser {

class UpsampleLayer {
public:
    explicit UpsampleLayer(int scale_factor = 2) : scale_factor_(scale_factor) {
        if (scale_factor <= 0) throw std::invalid_argument("UpsampleLayer: scale_factor must be > 0");
    }
    UpsampleLayer(const UpsampleLayer&) = delete;
    UpsampleLayer& operator=(const UpsampleLayer&) = delete;

    Tensor forward(const Tensor& input, cudaStream_t stream = nullptr) const {
        if (input.dtype() != DType::kFloat16) throw std::runtime_error("UpsampleLayer::forward: expected FP16 input");
        Tensor out = Tensor::empty({input.batch(), input.channels(), input.height() * scale_factor_,
                                    input.width() * scale_factor_},
                                   DType::kFloat16);
        detail::check(dn_upsample_bilinear(input.data(), out.data(), static_cast<int>(input.batch()),
                                           static_cast<int>(input.channels()), static_cast<int>(input.height()),
                                           static_cast<int>(input.width()), scale_factor_, stream));
        return out;
    }

    int scale_factor() const noexcept { return scale_factor_; }

private:
    int scale_factor_ = 2;
};

}  // namespace denoiser
