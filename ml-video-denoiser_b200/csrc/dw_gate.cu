// Depthwise 3x3 + bias + SimpleGate + global average pool + SCA, one pass.
//
// Reads the conv1 output u (NHWC, 2D channels), writes the gated tensor
// g = dw(u)[:D] * dw(u)[D:] (NHWC, D channels) and, per image, the
// simplified-channel-attention scale s = W_sca * mean_{HW}(g) + b_sca.
// The pool is a deterministic two-level reduction: each CTA writes its
// per-channel partial sums, and the last CTA of an image (atomic ticket)
// sums the partials in CTA order and evaluates the SCA 1x1 matvec.
//
// Replaces the reference's grouped cudnnConvolutionForward (conv2,
// src/models/nafnet.cu:126-130, 162), simple_gate_kernel, the serial
// global_avg_pool_kernel (one thread per channel looping over H*W),
// the SCA cudnn 1x1 on the pooled map and mul_channelwise's scale source
// (src/kernels/nafnet_kernels.cu:94-141).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kernels.h"
#include "sm100.cuh"
#include "status.h"

namespace dnb {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ void acc8(float (&a)[8], const uint4& v, const float* w) {
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = unpack_half2(u[i]);
        a[2 * i] += t.x * w[2 * i];
        a[2 * i + 1] += t.y * w[2 * i + 1];
    }
}

__global__ void __launch_bounds__(kThreads) dw_gate_sca_kernel(const __grid_constant__ DwParams p) {
    // Shared: taps [9][2D], bias [2D], then the pool reduction [lanes][D].
    extern __shared__ float sm[];
    __shared__ bool s_last;
    const int D = p.D;
    const int groups = D / 8;               // 8-channel groups of the gated output
    const int lanes = kThreads / groups;    // pixels processed concurrently
    const int tid = threadIdx.x;
    const int cg = tid % groups;
    const int pl = tid / groups;
    const int img = blockIdx.y;
    const int HW = p.H * p.W;
    const int C2 = 2 * D;
    float* sw = sm;
    float* sb = sm + 9 * C2;
    float* red = sb + C2;
    for (int i = tid; i < 9 * C2; i += kThreads) sw[i] = p.w[i];
    for (int i = tid; i < C2; i += kThreads) sb[i] = p.b[i];
    __syncthreads();
    const __half* u = p.u + static_cast<size_t>(img) * HW * C2;
    __half* g = p.g + static_cast<size_t>(img) * HW * D;
    const int c0 = cg * 8;

    float psum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (pl < lanes) {
        const int stride = lanes * gridDim.x;
        for (int pix = blockIdx.x * lanes + pl; pix < HW; pix += stride) {
            const int y = pix / p.W;
            const int x = pix - y * p.W;
            float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            float b[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
            for (int ky = 0; ky < 3; ++ky) {
                const int yy = y + ky - 1;
                if (yy < 0 || yy >= p.H) continue;
#pragma unroll
                for (int kx = 0; kx < 3; ++kx) {
                    const int xx = x + kx - 1;
                    if (xx < 0 || xx >= p.W) continue;
                    const __half* src = u + (static_cast<size_t>(yy) * p.W + xx) * C2;
                    const uint4 va = __ldg(reinterpret_cast<const uint4*>(src + c0));
                    const uint4 vb = __ldg(reinterpret_cast<const uint4*>(src + D + c0));
                    acc8(a, va, sw + (ky * 3 + kx) * C2 + c0);
                    acc8(b, vb, sw + (ky * 3 + kx) * C2 + D + c0);
                }
            }
            float o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = (a[i] + sb[c0 + i]) * (b[i] + sb[D + c0 + i]);
            uint4 ov;
            ov.x = pack_half2(o[0], o[1]);
            ov.y = pack_half2(o[2], o[3]);
            ov.z = pack_half2(o[4], o[5]);
            ov.w = pack_half2(o[6], o[7]);
            *reinterpret_cast<uint4*>(g + static_cast<size_t>(pix) * D + c0) = ov;
            // Pool the stored (fp16-rounded) values.
            const uint32_t q[4] = {ov.x, ov.y, ov.z, ov.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 t = unpack_half2(q[i]);
                psum[2 * i] += t.x;
                psum[2 * i + 1] += t.y;
            }
        }
    }

    // Block reduction over pixel lanes -> partials[img][block][D].
    if (pl < lanes) {
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
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned prev = atomicAdd(p.counter + img, 1u);
        s_last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;

    // Last CTA of this image: pool in CTA order, then the SCA matvec.
    __threadfence();
    float* mean = red;  // reuse: D floats
    const float inv = 1.0f / static_cast<float>(HW);
    for (int c = tid; c < D; c += kThreads) {
        const float* pp = p.partials + static_cast<size_t>(img) * gridDim.x * D + c;
        float s = 0.f;
        for (unsigned b = 0; b < gridDim.x; ++b) s += __ldcg(pp + static_cast<size_t>(b) * D);
        mean[c] = s * inv;
    }
    __syncthreads();
    const int warp = tid >> 5, lane = tid & 31;
    for (int o = warp; o < D; o += kThreads / 32) {
        const float* wr = p.sca_w + static_cast<size_t>(o) * D;
        float s = 0.f;
        for (int c = lane; c < D; c += 32) s += wr[c] * mean[c];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (lane == 0) p.s_out[static_cast<size_t>(img) * D + o] = s + p.sca_b[o];
    }
    if (tid == 0) p.counter[img] = 0u;
}

}  // namespace

int dw_blocks_per_img(int H, int W, int D) {
    const int lanes = kThreads / (D / 8);
    const long long px = static_cast<long long>(H) * W;
    long long blocks = (px + lanes * 8 - 1) / (lanes * 8);  // ~8 pixels per thread
    if (blocks < 1) blocks = 1;
    if (blocks > 148 * 8) blocks = 148 * 8;
    return static_cast<int>(blocks);
}

int launch_dw_gate_sca(const DwParams& p, int blocks_per_img, cudaStream_t s) {
    if (p.D % 8 != 0 || p.D / 8 > kThreads)
        return dn_fail(DN_ERR_UNSUPPORTED, "dw_gate: channels must be a multiple of 8 and <= 2048");
    const int lanes = kThreads / (p.D / 8);
    const size_t smem = (static_cast<size_t>(10) * 2 * p.D + static_cast<size_t>(lanes) * p.D) *
                        sizeof(float);
    if (smem > 200 * 1024) return dn_fail(DN_ERR_UNSUPPORTED, "dw_gate: too many channels");
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(dw_gate_sca_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return dn_cuda_fail(e, "dw_gate: set smem attribute");
        configured = true;
    }
    dim3 grid(blocks_per_img, p.N);
    dw_gate_sca_kernel<<<grid, kThreads, smem, s>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return dn_cuda_fail(e, "dw_gate: launch");
    return DN_OK;
}

}  // namespace dnb
