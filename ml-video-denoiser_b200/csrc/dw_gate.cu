// Depthwise 3x3 + bias + SimpleGate + global average pool, then the SCA
// matvec, as two kernels:
//
// dw_gate_kernel: reads the conv1 output u (NHWC, 2D channels), writes the
//   gated tensor g = dw(u)[:D] * dw(u)[D:] (NHWC, D channels) and per-CTA
//   per-channel partial sums of g. One thread computes one output pixel for
//   8 channels of both gate halves: its 18 tap loads are independent, the
//   tap weights are broadcast reads from shared memory.
// sca_kernel: each CTA re-reduces all partial sums of its image in a fixed
//   order (deterministic pool), then evaluates 8 outputs of
//   s = W_sca * mean_{HW}(g) + b_sca with coalesced weight-row reads.
//
// Replaces the reference's grouped cudnnConvolutionForward (conv2,
// src/models/nafnet.cu:126-130, 162), simple_gate_kernel, the serial
// global_avg_pool_kernel, the SCA cudnn 1x1 on the pooled map and
// mul_channelwise's scale source (src/kernels/nafnet_kernels.cu:94-141).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "kernels.h"
#include "launch.cuh"
#include "sm100.cuh"
#include "status.h"

namespace dnb {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ void fma8(float (&a)[8], const uint4& v, const float* w) {
    const float4 w0 = *reinterpret_cast<const float4*>(w);
    const float4 w1 = *reinterpret_cast<const float4*>(w + 4);
    const float2 t0 = unpack_half2(v.x), t1 = unpack_half2(v.y), t2 = unpack_half2(v.z), t3 = unpack_half2(v.w);
    a[0] = fmaf(t0.x, w0.x, a[0]);
    a[1] = fmaf(t0.y, w0.y, a[1]);
    a[2] = fmaf(t1.x, w0.z, a[2]);
    a[3] = fmaf(t1.y, w0.w, a[3]);
    a[4] = fmaf(t2.x, w1.x, a[4]);
    a[5] = fmaf(t2.y, w1.y, a[5]);
    a[6] = fmaf(t3.x, w1.z, a[6]);
    a[7] = fmaf(t3.y, w1.w, a[7]);
}

__global__ void __launch_bounds__(kThreads) dw_gate_kernel(const __grid_constant__ DwParams p) {
    // Shared: taps [9][2D], bias [2D], pool partials [lanes][D].
    extern __shared__ __align__(16) float sm[];
    const int D = p.D;
    const int C2 = 2 * D;
    const int groups = D / 8;
    const int lanes = kThreads / groups;  // pixels in flight per CTA
    const int tid = threadIdx.x;
    const int cg = tid % groups;
    const int pl = tid / groups;
    const int img = blockIdx.y;
    const int HW = p.H * p.W;
    float* sw = sm;
    float* sb = sw + 9 * C2;
    float* red = sb + C2;
    pdl_trigger();
    for (int i = tid; i < 9 * C2; i += kThreads) sw[i] = p.w[i];
    for (int i = tid; i < C2; i += kThreads) sb[i] = p.b[i];
    __syncthreads();
    pdl_wait();
    const __half* u = p.u + static_cast<size_t>(img) * HW * C2;
    __half* g = p.g + static_cast<size_t>(img) * HW * D;
    const int c0 = cg * 8;

    float psum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (pl < lanes) {
        const int stride = lanes * gridDim.x;
        for (int pix = blockIdx.x * lanes + pl; pix < HW; pix += stride) {
            const int y = pix / p.W;
            const int x = pix - y * p.W;
            uint4 va[9], vb[9];
#pragma unroll
            for (int t = 0; t < 9; ++t) {
                const int yy = y + t / 3 - 1, xx = x + t % 3 - 1;
                va[t] = make_uint4(0, 0, 0, 0);
                vb[t] = make_uint4(0, 0, 0, 0);
                if (yy >= 0 && yy < p.H && xx >= 0 && xx < p.W) {
                    const __half* src = u + (static_cast<size_t>(yy) * p.W + xx) * C2 + c0;
                    va[t] = __ldg(reinterpret_cast<const uint4*>(src));
                    vb[t] = __ldg(reinterpret_cast<const uint4*>(src + D));
                }
            }
            float a[8], b[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                a[i] = sb[c0 + i];
                b[i] = sb[D + c0 + i];
            }
#pragma unroll
            for (int t = 0; t < 9; ++t) {
                fma8(a, va[t], sw + t * C2 + c0);
                fma8(b, vb[t], sw + t * C2 + D + c0);
            }
            uint4 ov;
            ov.x = pack_half2(a[0] * b[0], a[1] * b[1]);
            ov.y = pack_half2(a[2] * b[2], a[3] * b[3]);
            ov.z = pack_half2(a[4] * b[4], a[5] * b[5]);
            ov.w = pack_half2(a[6] * b[6], a[7] * b[7]);
            *reinterpret_cast<uint4*>(g + static_cast<size_t>(pix) * D + c0) = ov;
            const uint32_t q[4] = {ov.x, ov.y, ov.z, ov.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 t = unpack_half2(q[i]);  // pool the stored fp16 values
                psum[2 * i] += t.x;
                psum[2 * i + 1] += t.y;
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) red[pl * D + c0 + i] = psum[i];
    }
    __syncthreads();
    float* part = p.partials + (static_cast<size_t>(img) * gridDim.x + blockIdx.x) * D;
    for (int c = tid; c < D; c += kThreads) {
        float s = 0.f;
        for (int l = 0; l < lanes; ++l) s += red[l * D + c];
        part[c] = s;
    }
}

// grid (D / 8, N): CTA j computes s[img][8j .. 8j+8). Every lane owns
// float4 channel vectors v = lane + 32 i (i < V, V = ceil(D / 128)); each
// phase issues all of its loads before it uses any, so it pays about one
// memory latency.
constexpr int kScaVec = 8;  // D <= 32 * 4 * kScaVec = 1024

template <int V>
__global__ void __launch_bounds__(kThreads) sca_kernel(const __grid_constant__ DwParams p, int nb) {
    constexpr int kScaVec = V;
    extern __shared__ __align__(16) float sm[];
    const int D = p.D;
    float* mean = sm;       // [D]
    float* red = sm + D;    // [stripes][D], stripes * D = 4 * kThreads floats
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int img = blockIdx.y;
    const int nvec = D / 4;
    pdl_trigger();
    // The weight row and bias of this warp's output (constant) load before the wait.
    const int o = blockIdx.x * 8 + warp;  // 8 warps -> 8 outputs
    const float bias_o = o < D ? p.sca_b[o] : 0.f;
    float4 w[kScaVec];
#pragma unroll
    for (int i = 0; i < kScaVec; ++i) {
        const int v = lane + 32 * i;
        w[i] = (o < D && v < nvec) ? reinterpret_cast<const float4*>(p.sca_w + static_cast<size_t>(o) * D)[v]
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // The conv3 B chunks this CTA rescales (constant weights) also load
    // before the wait: one 16-byte chunk (its 8 columns) of output rows
    // n = tid + u * kThreads.
    constexpr int kFold = 4;  // b_rows <= kFold * kThreads (checked at launch)
    const bool fold = p.bdst != nullptr;
    uint4 bv[kFold];
    size_t boff[kFold];
    if (fold) {
        const int k0 = blockIdx.x * 8;
        const int kc = k0 / p.b_kc, kq = (k0 % p.b_kc) / 8;
        const size_t tile_b = static_cast<size_t>(p.b_nt) * p.b_kc * 2;
        const uint32_t sbo = static_cast<uint32_t>(p.b_kc / 8) * 128u;
#pragma unroll
        for (int u = 0; u < kFold; ++u) {
            const int n = tid + u * kThreads;
            boff[u] = 0;
            bv[u] = make_uint4(0, 0, 0, 0);
            if (n < p.b_rows) {
                const int nt = n / p.b_nt, nl = n - nt * p.b_nt;
                boff[u] = (static_cast<size_t>(nt) * p.b_kchunks + kc) * tile_b + (nl >> 3) * sbo + kq * 128 +
                          (nl & 7) * 16;
                bv[u] = __ldg(reinterpret_cast<const uint4*>(p.bsrc + boff[u]));
            }
        }
    }
    pdl_wait();
    // Fixed-order pool over all 256 threads: thread (stripe, v) sums the
    // float4 channel vector v of partial rows stripe, stripe + stripes, ...
    // in row order; the stripe sums are then added in stripe order.
    const float4* pp = reinterpret_cast<const float4*>(p.partials + static_cast<size_t>(img) * nb * D);
    const int stripes = kThreads / nvec;
    const int v = tid % nvec, stripe = tid / nvec;
    if (stripe < stripes) {
        // Up to kPool rows in flight per thread (one memory latency for the
        // usual <= 12 rows per stripe), added in row order.
        constexpr int kPool = 12;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int b = stripe; b < nb; b += kPool * stripes) {
            float4 x[kPool];
#pragma unroll
            for (int u = 0; u < kPool; ++u) {
                const int row = min(b + u * stripes, nb - 1);  // past the end: a row that is not added
                x[u] = pp[static_cast<size_t>(row) * nvec + v];
            }
#pragma unroll
            for (int u = 0; u < kPool; ++u) {
                if (b + u * stripes < nb) {
                    acc.x += x[u].x;
                    acc.y += x[u].y;
                    acc.z += x[u].z;
                    acc.w += x[u].w;
                }
            }
        }
        reinterpret_cast<float4*>(red + stripe * D)[v] = acc;
    }
    __syncthreads();
    const float inv = 1.0f / static_cast<float>(p.H * p.W);
    for (int c = tid; c < D; c += kThreads) {
        float s = 0.f;
        for (int st = 0; st < stripes; ++st) s += red[st * D + c];
        mean[c] = s * inv;
    }
    __syncthreads();
    if (o < D) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < kScaVec; ++i) {
            const int v = lane + 32 * i;
            if (v < nvec) {
                const float4 m = reinterpret_cast<const float4*>(mean)[v];
                s = fmaf(w[i].x, m.x, s);
                s = fmaf(w[i].y, m.y, s);
                s = fmaf(w[i].z, m.z, s);
                s = fmaf(w[i].w, m.w, s);
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (lane == 0) p.s_out[static_cast<size_t>(img) * D + o] = s + bias_o;
        if (lane == 0) red[warp] = s + bias_o;  // red[] is no longer read: keep this CTA's s there
    }
    if (!fold) return;
    // Fold s[8j .. 8j+8) into the conv3 B columns of this CTA's 8 channels
    // (the chunks loaded before the wait).
    __syncthreads();
    const int k0 = blockIdx.x * 8;
    float sc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) sc[i] = (k0 + i < D) ? red[i] : 0.f;
#pragma unroll
    for (int u = 0; u < kFold; ++u) {
        if (tid + u * kThreads < p.b_rows) {
            float f[8];
            h8_to_f(bv[u], f);
#pragma unroll
            for (int i = 0; i < 8; ++i) f[i] *= sc[i];
            *reinterpret_cast<uint4*>(p.bdst + boff[u]) = f_to_h8(f);
        }
    }
}

}  // namespace

int dw_blocks_per_img(int H, int W, int D) {
    const int lanes = kThreads / (D / 8 > kThreads ? kThreads : D / 8);
    const long long px = static_cast<long long>(H) * W;
    const long long want = (px + lanes * 4 - 1) / (lanes * 4);  // ~4 pixels per thread
    // The SCA pool re-reads nb x D partials per CTA: keep nb x D modest.
    const long long cap = std::max(148LL, std::min(148LL * 4, 148LL * 4 * 64 / std::max(D, 64)));
    return static_cast<int>(std::max(1LL, std::min(want, cap)));
}

template <int V>
int launch_sca_v(const DwParams& p, int nb, cudaStream_t s) {
    const size_t smem = (static_cast<size_t>(p.D) + 4 * kThreads) * sizeof(float);
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(sca_kernel<V>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
        if (e != cudaSuccess) return dn_cuda_fail(e, "sca: set smem attribute");
        configured = true;
    }
    cudaError_t e = launch_pdl(sca_kernel<V>, dim3((p.D + 7) / 8, p.N), dim3(kThreads), smem, s, p, nb);
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "sca: launch");
}

int launch_sca(const DwParams& p, int nb, cudaStream_t s) {
    if (p.D % 4 != 0 || p.D > 32 * 4 * kScaVec)
        return dn_fail(DN_ERR_UNSUPPORTED, "sca: channels must be a multiple of 4 and <= 1024");
    if (p.bdst && p.b_rows > 4 * kThreads)
        return dn_fail(DN_ERR_UNSUPPORTED, "sca: conv3 has more than 1024 output channels");
    const int nvec = p.D / 4;
    if (nvec <= 32) return launch_sca_v<1>(p, nb, s);
    if (nvec <= 64) return launch_sca_v<2>(p, nb, s);
    if (nvec <= 128) return launch_sca_v<4>(p, nb, s);
    return launch_sca_v<8>(p, nb, s);
}

int launch_dw_gate_sca(const DwParams& p, int blocks_per_img, cudaStream_t s) {
    if (p.D % 8 != 0 || p.D > 32 * 4 * kScaVec)
        return dn_fail(DN_ERR_UNSUPPORTED, "dw_gate: channels must be a multiple of 8 and <= 1024");
    const int lanes = kThreads / (p.D / 8);
    const size_t smem = (static_cast<size_t>(10) * 2 * p.D + static_cast<size_t>(lanes) * p.D) * sizeof(float);
    const size_t smem2 = static_cast<size_t>(9) * p.D * sizeof(float);
    if (smem > 200 * 1024 || smem2 > 200 * 1024) return dn_fail(DN_ERR_UNSUPPORTED, "dw_gate: too many channels");
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(dw_gate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return dn_cuda_fail(e, "dw_gate: set smem attribute");
        configured = true;
    }
    cudaError_t e = launch_pdl(dw_gate_kernel, dim3(blocks_per_img, p.N), dim3(kThreads), smem, s, p);
    if (e != cudaSuccess) return dn_cuda_fail(e, "dw_gate: launch");
    return launch_sca(p, blocks_per_img, s);
}

}  // namespace dnb
