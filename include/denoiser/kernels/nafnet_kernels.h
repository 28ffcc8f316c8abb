// denoiser::kernels launchers of the reference's
// include/denoiser/kernels/nafnet_kernels.h:9-95 (same signatures), over
// include/denoiser_b200_ops.h. Arguments the reference would read out of
// bounds with throw std::invalid_argument; CUDA failures std::runtime_error.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "denoiser/detail/abi.h"
#include "denoiser_b200_ops.h"

namespace denoiser::kernels {

inline void launch_extract_frame(const __half* clip, __half* frame, int N, int T, int C, int H, int W, int frame_idx,
                                 cudaStream_t stream) {
    detail::check(dn_launch_extract_frame(clip, frame, N, T, C, H, W, frame_idx, stream));
}

inline void launch_select_prefix_channels(const __half* input, __half* output, int N, int C_in, int C_out, int H, int W,
                                          cudaStream_t stream) {
    detail::check(dn_launch_select_prefix_channels(input, output, N, C_in, C_out, H, W, stream));
}

inline void launch_layer_norm_affine(const __half* input, const void* weight, const void* bias, bool params_fp32,
                                     __half* output, int N, int C, int H, int W, cudaStream_t stream) {
    detail::check(dn_launch_layer_norm_affine(input, weight, bias, params_fp32 ? 1 : 0, output, N, C, H, W, stream));
}

inline void launch_simple_gate(const __half* input, __half* output, int N, int C, int H, int W, cudaStream_t stream) {
    detail::check(dn_launch_simple_gate(input, output, N, C, H, W, stream));
}

inline void launch_global_avg_pool(const __half* input, __half* output, int N, int C, int H, int W, cudaStream_t stream) {
    detail::check(dn_launch_global_avg_pool(input, output, N, C, H, W, stream));
}

inline void launch_mul_channelwise(const __half* input, const __half* scale, __half* output, int N, int C, int H, int W,
                                   cudaStream_t stream) {
    detail::check(dn_launch_mul_channelwise(input, scale, output, N, C, H, W, stream));
}

inline void launch_add(const __half* a, const __half* b, __half* out, int64_t n, cudaStream_t stream) {
    detail::check(dn_launch_add(a, b, out, n, stream));
}

inline void launch_mul_scalar(const __half* input, float scalar, __half* output, int64_t n, cudaStream_t stream) {
    detail::check(dn_launch_mul_scalar(input, scalar, output, n, stream));
}

inline void launch_scaled_add(const __half* identity, const __half* residual, const void* scale, bool scale_fp32,
                              __half* output, int N, int C, int H, int W, cudaStream_t stream) {
    detail::check(dn_launch_scaled_add(identity, residual, scale, scale_fp32 ? 1 : 0, output, N, C, H, W, stream));
}

inline void launch_pixel_shuffle2x(const __half* input, __half* output, int N, int C_in, int H, int W,
                                   cudaStream_t stream) {
    detail::check(dn_launch_pixel_shuffle2x(input, output, N, C_in, H, W, stream));
}

inline void launch_warp_bilinear(const __half* feat, const __half* offset, __half* output, int N, int C, int H, int W,
                                 cudaStream_t stream) {
    detail::check(dn_launch_warp_bilinear(feat, offset, output, N, C, H, W, stream));
}

}  // namespace denoiser::kernels
