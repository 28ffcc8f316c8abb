// Fused NAFBlock kernels: both passes for the shallow levels (C <= 64,
// fused_block.cu) and the second pass for the deep levels (C = 128 / 256,
// deep_block.cu).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace dnb {

struct FusedAParams {
    const __half* x;        // block input, NHWC [N, H, W, C]
    __half* g;              // gated output, NHWC [N, H, W, D]
    int N, H, W;
    const uint8_t* w1;      // conv1 B = fp16(gamma1 * W1), one NT = 2D tile image
    const float* c1;        // [2D] sum_k B[n, k]
    const float* c2;        // [2D] bias1 + sum_k beta1[k] W1[n, k]
    const float* dw_w;      // [9][2D]
    const float* dw_b;      // [2D]
    float* partials;        // [N][grid][D] pool partial sums
    uint32_t* err;
    // Tensor-core form (fused_a_tc.cu): LN + conv1 + depthwise as one 3x3 conv.
    const uint8_t* weff;    // [3 kx][C/16 K steps][ky = 2, 1, 0] B tiles of Weff = dw * W1 * gamma1 (2D x 16 each)
    const float* b1p;       // [2D] b1 + W1 beta1
    // Single image (tensor-core form): the last CTA to finish reduces the pool
    // partials, evaluates the SCA and writes conv3's B with the scale folded
    // in (b3_dst = b3_src, column k times s[k]; one [C x D] tile, KC = D);
    // counter is zero on entry and reset by that CTA. b3_dst == nullptr: off.
    unsigned* counter;
    const float* sca_w;     // [D][D]
    const float* sca_b;     // [D]
    const uint8_t* b3_src;
    uint8_t* b3_dst;
};

struct FusedBParams {
    const __half* g;        // [M, D]
    const __half* x;        // [M, C] block input (residual)
    __half* out;            // [M, C]
    int M, hw;
    const float* s;         // SCA scale [N][D]; nullptr: already folded into w3 by the SCA kernel
    const uint8_t* w3;      // [C x D] tile image
    const uint8_t* w4;      // [2F x C] tile image (gate halves in order)
    const uint8_t* w5;      // [C x F] tile image
    const float *b3, *beta, *ln_w, *ln_b, *b4, *b5, *gamma;
    uint32_t* err;
};

bool fused_supported(int C, int D, int F);
bool fused_a_tc_supported(int C, int D);
int fused_a_tc_grid(int C, int N, int H, int W);
int launch_fused_a_tc(const FusedAParams& p, int C, int D, int grid, cudaStream_t s);
// Phase A with conv1 on the tensor cores and the depthwise conv on the CUDA
// cores (fused_a_split.cu): single image, C = D = 32 / 64; uses w1, c2,
// dw_w, dw_b, partials and the SCA fold fields.
bool fused_a_split_supported(int C, int D, int N);
int fused_a_split_grid(int C, int H, int W);
int launch_fused_a_split(const FusedAParams& p, int C, int D, int grid, cudaStream_t s);
int fused_a_grid(int C, int D, int N, int H, int W);
int launch_fused_a(const FusedAParams& p, int C, int D, int grid, cudaStream_t s);
int launch_fused_b(const FusedBParams& p, int C, int D, int F, cudaStream_t s);

// Second pass of a deep NAFBlock on one image, in place on x:
// y = x + beta * (g (W3 diag(s))^T + b3); h = SimpleGate(LN2(y) W4^T + b4);
// out = y + gamma * (h W5^T + b5), for C = D = F = 128 or 256. The B operands
// are the engine's tile images (K chunks of 64): w3 = the SCA-scaled conv3
// image ([C x D], one N tile), w4 = conv4 with LN2 folded as 128-row tiles
// [64 a rows | 64 b rows] per 64-channel gate chunk (c1, c2 in that packed
// order), w5 = conv5 ([C x F], one N tile).
struct DeepBParams {
    const __half* g;        // [M, D]
    const __half* x;        // [M, C]
    __half* out;            // [M, C] (may alias x)
    int M;
    const uint8_t *w3, *w4, *w5;
    const float *b3, *beta, *c1, *c2, *b5, *gamma;
    uint32_t* err;
};

bool deep_b_supported(int C, int D, int F);
int launch_deep_b(const DeepBParams& p, int C, int D, int F, cudaStream_t s);

// Shared host helpers: FP16 tensor map (tiled, no interleave, L2 promotion
// 128 B, zero fill) and the device's SM count.
int encode_f16_map(CUtensorMap* m, int rank, const void* base, const cuuint64_t* dims, const cuuint64_t* strides,
                   const cuuint32_t* box, CUtensorMapSwizzle swz);
int sm_count();

}  // namespace dnb
