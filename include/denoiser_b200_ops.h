/*
 * denoiser_b200_ops.h — C-ABI of the NCHW FP16 kernel launchers.
 *
 * One entry point per reference launcher in denoiser::kernels
 * (include/denoiser/kernels/model_kernels.h:22-59 and
 * include/denoiser/kernels/nafnet_kernels.h:9-95 of the reference), with the
 * same argument order and meaning. Tensor pointers are device pointers to
 * IEEE binary16 (__half) data in contiguous NCHW order; `stream` is a
 * cudaStream_t (NULL = legacy default stream). Work is enqueued
 * asynchronously on `stream`.
 *
 * Differences from the reference launchers, which return void:
 *   - every function returns DN_OK or a negative DN_ERR_* code (see
 *     denoiser_b200.h) and never throws; dn_last_error() has the message;
 *   - arguments the reference would turn into out-of-bounds accesses
 *     (negative sizes, a reflect pad wider than the image, a crop larger than
 *     its input, a frame index outside the clip, C_in not divisible by 4 for
 *     the pixel shuffle) are rejected with DN_ERR_INVALID_ARG;
 *   - a size of zero elements is a successful no-op.
 * The C++ headers under include/denoiser/kernels/ wrap these back into the
 * reference's void launch_* signatures, throwing std::runtime_error.
 */
#ifndef DENOISER_B200_OPS_H
#define DENOISER_B200_OPS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* launch_reflect_pad (model_kernels.h:22): output (N,C,H_out,W_out) from
 * input (N,C,H_in,W_in), reflecting at the bottom/right edge:
 * h >= H_in -> 2*(H_in-1) - h (same for w). Requires H_in <= H_out <= 2*H_in-1
 * and W_in <= W_out <= 2*W_in-1. */
int dn_launch_reflect_pad(const void* input, void* output, int N, int C, int H_in, int W_in, int H_out,
                          int W_out, void* stream);

/* launch_crop (model_kernels.h:34): the top-left (N,C,H_out,W_out) corner of
 * input (N,C,H_in,W_in). Requires H_out <= H_in and W_out <= W_in. */
int dn_launch_crop(const void* input, void* output, int N, int C, int H_in, int W_in, int H_out, int W_out,
                   void* stream);

/* launch_subtract_clamp (model_kernels.h:45): out[i] = clamp(a[i] - b[i], 0, 1). */
int dn_launch_subtract_clamp(const void* a, const void* b, void* out, int64_t n, void* stream);

/* launch_concat_channels (model_kernels.h:53): output (N,C1+C2,H,W) =
 * [a (N,C1,H,W), b (N,C2,H,W)] along channels. */
int dn_launch_concat_channels(const void* a, const void* b, void* output, int N, int C1, int C2, int H, int W,
                              void* stream);

/* launch_extract_frame (nafnet_kernels.h:9): frame (N,C,H,W) = clip[:, frame_idx]
 * of clip (N,T,C,H,W). Requires 0 <= frame_idx < T. */
int dn_launch_extract_frame(const void* clip, void* frame, int N, int T, int C, int H, int W, int frame_idx,
                            void* stream);

/* launch_select_prefix_channels (nafnet_kernels.h:16): output (N,C_out,H,W) =
 * the first C_out channels of input (N,C_in,H,W). Requires C_out <= C_in. */
int dn_launch_select_prefix_channels(const void* input, void* output, int N, int C_in, int C_out, int H, int W,
                                     void* stream);

/* launch_layer_norm_affine (nafnet_kernels.h:23): per pixel, normalise over
 * the C channels (biased variance, eps 1e-6, FP32 statistics), then
 * * weight[c] + bias[c]. weight/bias are FP32 when params_fp32 != 0, else FP16.
 * Supports C <= 2048. */
int dn_launch_layer_norm_affine(const void* input, const void* weight, const void* bias, int params_fp32,
                                void* output, int N, int C, int H, int W, void* stream);

/* launch_simple_gate (nafnet_kernels.h:33): output (N,C,H,W) = x1 * x2 where
 * x1, x2 are the two channel halves of input (N,2C,H,W) of each image. (The
 * reference kernel indexes the input as if N were 1; both agree for N == 1.) */
int dn_launch_simple_gate(const void* input, void* output, int N, int C, int H, int W, void* stream);

/* launch_global_avg_pool (nafnet_kernels.h:40): output (N,C) FP16 = the mean
 * over H*W of each plane of input (N,C,H,W), accumulated in FP32. Each plane is
 * split across thread blocks and the per-block sums are added in a fixed
 * order, so results are deterministic. The per-call FP32 scratch of the
 * split sums (N*C*splits floats, splits <= 128) is allocated and freed on
 * `stream` (cudaMallocAsync / cudaFreeAsync). */
int dn_launch_global_avg_pool(const void* input, void* output, int N, int C, int H, int W, void* stream);

/* dn_launch_global_avg_pool without any device allocation (no counterpart in
 * the reference). For callers that must not allocate device memory: host
 * applications that have reserved the GPU's memory for their own pool, where
 * an allocation fails or evicts their cache, and per-frame real-time loops,
 * where cudaMalloc/cudaFree stall the device mid-frame. The split sums go to
 * a fixed 1 MiB array in this library's device code instead:
 *   - limit: N*C*splits <= 262144, splits = min(128, ceil(H*W / 16384)), so
 *     any N*C <= 2048 fits; larger sizes return DN_ERR_UNSUPPORTED;
 *   - the first call on each device (with that device current) looks up the
 *     array's device address once; make that first call before any stream
 *     capture begins. The looked-up address is kept for the life of the
 *     process and does not survive cudaDeviceReset: do not call this entry
 *     point on a device after resetting it;
 *   - a size beyond the limit is rejected on the host before any CUDA call;
 *   - the array is shared by every call on the device: calls whose work may
 *     overlap on the GPU (different streams without an event between them,
 *     or concurrent host threads) race on it and give wrong means. Order
 *     them on one stream.
 * Results equal dn_launch_global_avg_pool's (same plan and kernels). */
int dn_launch_global_avg_pool_noalloc(const void* input, void* output, int N, int C, int H, int W, void* stream);

/* launch_mul_channelwise (nafnet_kernels.h:47): output = input * scale[n*C + c],
 * scale (N,C) FP16. */
int dn_launch_mul_channelwise(const void* input, const void* scale, void* output, int N, int C, int H, int W,
                              void* stream);

/* launch_add (nafnet_kernels.h:55): out[i] = a[i] + b[i]. */
int dn_launch_add(const void* a, const void* b, void* out, int64_t n, void* stream);

/* launch_mul_scalar (nafnet_kernels.h:63): output[i] = input[i] * scalar. */
int dn_launch_mul_scalar(const void* input, float scalar, void* output, int64_t n, void* stream);

/* launch_scaled_add (nafnet_kernels.h:71): output = identity + residual * scale[c],
 * scale (C) FP32 when scale_fp32 != 0, else FP16. */
int dn_launch_scaled_add(const void* identity, const void* residual, const void* scale, int scale_fp32,
                         void* output, int N, int C, int H, int W, void* stream);

/* launch_pixel_shuffle2x (nafnet_kernels.h:81): PixelShuffle(2) of input
 * (N,C_in,H,W) into (N,C_in/4,2H,2W). Requires C_in % 4 == 0. */
int dn_launch_pixel_shuffle2x(const void* input, void* output, int N, int C_in, int H, int W, void* stream);

/* launch_warp_bilinear (nafnet_kernels.h:88): output (N,C,H,W) = feat sampled
 * at (w + dx, h + dy), bilinear, border-clamped, with offset (N,2,H,W) in
 * pixels (channel 0 = dx, channel 1 = dy). */
int dn_launch_warp_bilinear(const void* feat, const void* offset, void* output, int N, int C, int H, int W,
                            void* stream);

/* UpsampleLayer::forward (include/denoiser/layers/upsample.h:19-26): output
 * (N,C,H*s,W*s) = bilinear upsampling of input (N,C,H,W) by the integer
 * factor s = scale_factor, with the reference kernel's coordinate rule
 * (src/layers/upsample.cu:10-45): source (o + 0.5)/s - 0.5, low corner
 * clamped to 0 with the weight from the unclamped coordinate, high corner
 * clamped to the edge. DN_ERR_INVALID_ARG for scale_factor <= 0 (the
 * reference throws std::invalid_argument). */
int dn_upsample_bilinear(const void* input, void* output, int N, int C, int H, int W, int scale_factor,
                         void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DENOISER_B200_OPS_H */
