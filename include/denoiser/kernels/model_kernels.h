// denoiser::kernels launchers of the reference's
// include/denoiser/kernels/model_kernels.h:22-59 (same signatures), over
// include/denoiser_b200_ops.h. Arguments the reference would read out of
// bounds with throw std::invalid_argument; CUDA failures std::runtime_error.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "denoiser/detail/abi.h"
#include "denoiser_b200_ops.h"

namespace denoiser::kernels {

inline void launch_reflect_pad(const __half* input, __half* output, int N, int C, int H_in, int W_in, int H_out,
                               int W_out, cudaStream_t stream) {
    detail::check(dn_launch_reflect_pad(input, output, N, C, H_in, W_in, H_out, W_out, stream));
}

inline void launch_crop(const __half* input, __half* output, int N, int C, int H_in, int W_in, int H_out, int W_out,
                        cudaStream_t stream) {
    detail::check(dn_launch_crop(input, output, N, C, H_in, W_in, H_out, W_out, stream));
}

inline void launch_subtract_clamp(const __half* a, const __half* b, __half* out, int64_t n, cudaStream_t stream) {
    detail::check(dn_launch_subtract_clamp(a, b, out, n, stream));
}

inline void launch_concat_channels(const __half* a, const __half* b, __half* output, int N, int C1, int C2, int H,
                                   int W, cudaStream_t stream) {
    detail::check(dn_launch_concat_channels(a, b, output, N, C1, C2, H, W, stream));
}

}  // namespace denoiser::kernels
