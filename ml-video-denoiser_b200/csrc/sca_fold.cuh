// The SCA of a single-image NAFBlock, evaluated by the last CTA of the
// kernel that produced the pool partials (the first pass of a 32/64-channel
// block), with the channel scale folded into conv3's B operand:
//   mean[c] = (sum over the CTAs' partial rows, fixed order) / (H * W)
//   s       = W_sca mean + b_sca                 (sca.1, a 1x1 conv on the pool)
//   B3'     = B3 diag(s)                          (conv3's columns scaled by s)
// which replaces the reference's global_avg_pool_kernel, the sca 1x1
// cudnnConvolutionForward and mul_channelwise_kernel
// (src/models/nafnet.cu:174-188, src/kernels/nafnet_kernels.cu:108-141).
//
// Every CTA calls it after its partial row is in global memory; an atomic
// counter (zero on entry, reset by the last CTA) elects the last one. Each
// phase issues all of its loads before it uses any: the constant SCA
// weights and conv3 B chunks first, then the CTAs' pool rows.
#pragma once

#include <cuda_fp16.h>

#include "sm100.cuh"

namespace dnb {

// P: p.partials [grid][D], p.H, p.W, p.counter, p.sca_w [D][D], p.sca_b [D],
// p.b3_src / p.b3_dst (conv3 B image, C rows of D channels, one K chunk).
// scratch: at least 18 * D floats of shared memory no other role still uses.
template <int C, int D, int kThreads, class P>
__device__ __forceinline__ void sca_fold_last_cta(const P& p, float* scratch, int tid, int warp, int lane) {
    __shared__ int s_last;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(p.counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    constexpr int kWarps = kThreads / 32;
    constexpr int kOut = (D + kWarps - 1) / kWarps;  // SCA outputs per warp
    constexpr int kCol = D / 32;                     // weight columns per lane
    constexpr int KQ = D / 8;                        // 16-byte chunks per B row
    constexpr int kChunks = C * KQ;
    constexpr int kPer = (kChunks + kThreads - 1) / kThreads;
    float wv[kOut][kCol], bo[kOut];
#pragma unroll
    for (int j = 0; j < kOut; ++j) {
        const int o = warp + kWarps * j;
        bo[j] = o < D ? __ldg(p.sca_b + o) : 0.f;
#pragma unroll
        for (int i = 0; i < kCol; ++i) wv[j][i] = o < D ? __ldg(p.sca_w + o * D + lane + 32 * i) : 0.f;
    }
    uint4 bv[kPer];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
        const int i = tid + u * kThreads;
        const int n = i / KQ, q = i - n * KQ;
        bv[u] = i < kChunks ? __ldg(reinterpret_cast<const uint4*>(p.b3_src + static_cast<size_t>(n >> 3) * (KQ * 128) +
                                                                   q * 128 + (n & 7) * 16))
                            : make_uint4(0, 0, 0, 0);
    }
    // Fixed-order pool: thread (stripe, c) sums rows stripe, stripe + stripes,
    // ... of channel c; the stripes add in order.
    constexpr int kStripes = (kThreads / D) < 16 ? (kThreads / D) : 16;
    constexpr int kPool = 16;
    float* s_red = scratch;             // [kStripes][D]
    float* s_mean = scratch + 16 * D;   // [D]
    float* s_scale = s_mean + D;        // [D]
    const unsigned nb = gridDim.x;
    {
        const int c = tid % D, st = tid / D;
        if (st < kStripes) {
            float sum = 0.f;
            for (unsigned r0 = st; r0 < nb; r0 += kPool * kStripes) {
                float v[kPool];
#pragma unroll
                for (int u = 0; u < kPool; ++u) {
                    const unsigned r = min(r0 + u * kStripes, nb - 1);  // past the end: not added
                    v[u] = __ldcg(p.partials + static_cast<size_t>(r) * D + c);
                }
#pragma unroll
                for (int u = 0; u < kPool; ++u)
                    if (r0 + u * kStripes < nb) sum += v[u];
            }
            s_red[st * D + c] = sum;
        }
    }
    __syncthreads();
    const float inv = 1.0f / (static_cast<float>(p.H) * p.W);
    for (int c = tid; c < D; c += kThreads) {
        float sum = 0.f;
        for (int st = 0; st < kStripes; ++st) sum += s_red[st * D + c];
        s_mean[c] = sum * inv;
    }
    __syncthreads();
    // s = W mean + b: warp w evaluates outputs w, w + kWarps, ...
#pragma unroll
    for (int j = 0; j < kOut; ++j) {
        const int o = warp + kWarps * j;
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < kCol; ++i) acc = fmaf(wv[j][i], s_mean[lane + 32 * i], acc);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (lane == 0 && o < D) s_scale[o] = acc + bo[j];
    }
    __syncthreads();
    // conv3's B columns scaled by s.
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
        const int i = tid + u * kThreads;
        if (i < kChunks) {
            const int n = i / KQ, q = i - n * KQ;
            float f[8];
            h8_to_f(bv[u], f);
#pragma unroll
            for (int j = 0; j < 8; ++j) f[j] *= s_scale[8 * q + j];
            *reinterpret_cast<uint4*>(p.b3_dst + static_cast<size_t>(n >> 3) * (KQ * 128) + q * 128 + (n & 7) * 16) =
                f_to_h8(f);
        }
    }
    if (tid == 0) *p.counter = 0u;
}

}  // namespace dnb
