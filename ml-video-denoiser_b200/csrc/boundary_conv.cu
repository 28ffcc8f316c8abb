// The two dense 3x3 convolutions at the network boundary, on CUDA cores
// (N = 32 output channels from K = 27 inputs for the intro, N = 3 outputs
// for the ending: too narrow for a 128-row tensor-core tile to pay off).
//
// intro  : replaces select_beauty / reflect_pad_kernel / the intro cuDNN conv
//          + bias pass (src/models/nafnet.cu:354-357, src/kernels/model_kernels.cu
//          :15-34). Applies nan_to_num (training/models.py:559) and the
//          right/bottom reflect pad (h >= H -> 2(H-1) - h) while staging the tile.
// ending : replaces the ending cuDNN conv + bias, the unpad crop and the
//          beauty add (src/models/nafnet.cu:386-388): reads the NHWC features,
//          writes the cropped NCHW fp16 frame = beauty + residual.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kernels.h"
#include "launch.cuh"
#include "sm100.cuh"
#include "status.h"

namespace dnb {
namespace {

constexpr int kTile = 16;  // 16x16 output pixels per CTA, 256 threads

__device__ __forceinline__ float finite_or_zero(float v) {
    return (isnan(v) || isinf(v)) ? 0.f : v;
}

__device__ __forceinline__ int reflect_hi(int i, int n) { return i < n ? i : 2 * (n - 1) - i; }

__device__ __forceinline__ void h8_to_f(const uint4& v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = unpack_half2(w[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

// One thread = one output pixel, all C0 outputs (in groups of 8).
__global__ void __launch_bounds__(256) intro_kernel(const __grid_constant__ IntroParams p) {
    extern __shared__ float sm[];
    const int Cin = p.Cin, C0 = p.C0;
    float* sx = sm;                                   // [Cin][18][18]
    float* sw = sx + Cin * (kTile + 2) * (kTile + 2);  // [C0][Kp] (Kp = Cin*9 rounded to 4)
    const int img = blockIdx.z;
    const int ty0 = blockIdx.y * kTile, tx0 = blockIdx.x * kTile;
    const __half* x = p.x + static_cast<size_t>(img) * p.in_batch_stride;
    const int tid = threadIdx.x;
    const int K = Cin * 9;
    const int Kp = (K + 3) & ~3;
    pdl_trigger();
    for (int i = tid; i < C0 * Kp; i += 256) {
        const int o = i / Kp, k = i - o * Kp;
        sw[i] = k < K ? p.w[o * K + k] : 0.f;
    }
    pdl_wait();
    const int area = (kTile + 2) * (kTile + 2);
    for (int i = tid; i < Cin * area; i += 256) {
        const int c = i / area;
        const int r = i - c * area;
        const int yy = ty0 + r / (kTile + 2) - 1;  // coordinate in the padded frame
        const int xx = tx0 + r % (kTile + 2) - 1;
        float v = 0.f;  // conv zero padding outside the padded frame
        if (yy >= 0 && yy < p.Hp && xx >= 0 && xx < p.Wp) {
            const int sy = reflect_hi(yy, p.H);
            const int sx2 = reflect_hi(xx, p.W);
            v = finite_or_zero(__half2float(x[(static_cast<size_t>(c) * p.H + sy) * p.W + sx2]));
        }
        sx[i] = v;
    }
    __syncthreads();
    const int ly = tid / kTile, lx = tid % kTile;
    const int oy = ty0 + ly, ox = tx0 + lx;
    if (oy >= p.Hp || ox >= p.Wp) return;
    __half* dst = p.y + ((static_cast<size_t>(img) * p.Hp + oy) * p.Wp + ox) * C0;
    // The patch (Cin x 3 x 3) in registers; weight rows are broadcast reads.
    constexpr int kMaxK = 36;  // up to 4 input channels per pass
    for (int cbase = 0; cbase < Cin; cbase += 4) {
        const int cn = min(4, Cin - cbase);
        float v[kMaxK];
#pragma unroll
        for (int i = 0; i < kMaxK; ++i) {
            const int c = cbase + i / 9;
            const int t = i % 9;
            v[i] = (i < cn * 9) ? sx[c * area + (ly + t / 3) * (kTile + 2) + lx + t % 3] : 0.f;
        }
        for (int o0 = 0; o0 < C0; o0 += 8) {
            float acc[8];
            if (cbase == 0) {
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[i] = p.b[o0 + i];
            } else {
                float prev[8];
                h8_to_f(*reinterpret_cast<const uint4*>(dst + o0), prev);
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[i] = prev[i];
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                // cbase * 9 is a multiple of 4: 16-byte aligned broadcast reads.
                const float4* wr = reinterpret_cast<const float4*>(sw + (o0 + i) * Kp + cbase * 9);
#pragma unroll
                for (int k4 = 0; k4 < kMaxK / 4; ++k4) {
                    if (4 * k4 >= cn * 9) break;
                    const float4 w4 = wr[k4];
                    acc[i] = fmaf(v[4 * k4], w4.x, acc[i]);
                    acc[i] = fmaf(v[4 * k4 + 1], w4.y, acc[i]);
                    acc[i] = fmaf(v[4 * k4 + 2], w4.z, acc[i]);
                    acc[i] = fmaf(v[4 * k4 + 3], w4.w, acc[i]);
                }
            }
            uint4 ov;
            ov.x = pack_half2(acc[0], acc[1]);
            ov.y = pack_half2(acc[2], acc[3]);
            ov.z = pack_half2(acc[4], acc[5]);
            ov.w = pack_half2(acc[6], acc[7]);
            *reinterpret_cast<uint4*>(dst + o0) = ov;
        }
    }
}

// One thread = one output pixel of the cropped frame, 3 outputs.
__global__ void __launch_bounds__(256) ending_kernel(const __grid_constant__ EndingParams p) {
    extern __shared__ float sm[];
    const int C0 = p.C0;
    const int area = (kTile + 2) * (kTile + 2);
    float* sw = sm;               // [3][9][C0]
    // NHWC tile with a padded pixel stride (C0 + 2 halves: an odd number of
    // 32-bit words) so that lanes on neighbouring pixels hit distinct banks.
    const int ps = C0 + 2;
    __half* sx = reinterpret_cast<__half*>(sw + 27 * C0);  // [18*18][ps]
    const int img = blockIdx.z;
    const int ty0 = blockIdx.y * kTile, tx0 = blockIdx.x * kTile;
    const int tid = threadIdx.x;
    pdl_trigger();
    for (int i = tid; i < 27 * C0; i += 256) sw[i] = p.w[i];
    pdl_wait();
    const __half* xin = p.x + static_cast<size_t>(img) * p.Hp * p.Wp * C0;
    const int vec = C0 / 8;
    for (int i = tid; i < area * vec; i += 256) {
        const int r = i / vec;
        const int q = i - r * vec;
        const int yy = ty0 + r / (kTile + 2) - 1;
        const int xx = tx0 + r % (kTile + 2) - 1;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (yy >= 0 && yy < p.Hp && xx >= 0 && xx < p.Wp)
            v = __ldg(reinterpret_cast<const uint4*>(xin + (static_cast<size_t>(yy) * p.Wp + xx) * C0) + q);
        uint32_t* d = reinterpret_cast<uint32_t*>(sx + static_cast<size_t>(r) * ps + q * 8);
        d[0] = v.x;
        d[1] = v.y;
        d[2] = v.z;
        d[3] = v.w;
    }
    __syncthreads();
    const int ly = tid / kTile, lx = tid % kTile;
    const int oy = ty0 + ly, ox = tx0 + lx;
    if (oy >= p.H || ox >= p.W) return;
    float acc[3] = {p.b[0], p.b[1], p.b[2]};
#pragma unroll
    for (int ky = 0; ky < 3; ++ky)
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
            const __half* px = sx + static_cast<size_t>((ly + ky) * (kTile + 2) + lx + kx) * ps;
            const float* w0 = sw + (0 * 9 + ky * 3 + kx) * C0;
            const float* w1 = sw + (1 * 9 + ky * 3 + kx) * C0;
            const float* w2 = sw + (2 * 9 + ky * 3 + kx) * C0;
            for (int c = 0; c < C0; c += 2) {
                const float2 v = __half22float2(*reinterpret_cast<const __half2*>(px + c));
                acc[0] += v.x * w0[c] + v.y * w0[c + 1];
                acc[1] += v.x * w1[c] + v.y * w1[c + 1];
                acc[2] += v.x * w2[c] + v.y * w2[c + 1];
            }
        }
    const size_t plane = static_cast<size_t>(p.H) * p.W;
    const __half* beauty = p.beauty + static_cast<size_t>(img) * p.beauty_batch_stride;
    __half* out = p.y + static_cast<size_t>(img) * 3 * plane;
    const size_t o = static_cast<size_t>(oy) * p.W + ox;
#pragma unroll
    for (int c = 0; c < 3; ++c)
        out[c * plane + o] = __float2half(finite_or_zero(__half2float(beauty[c * plane + o])) + acc[c]);
}

}  // namespace

int launch_intro(const IntroParams& p, cudaStream_t s) {
    if (p.C0 % 8 != 0) return dn_fail(DN_ERR_UNSUPPORTED, "intro: base channels must be a multiple of 8");
    const size_t smem = (static_cast<size_t>(p.Cin) * (kTile + 2) * (kTile + 2) +
                         static_cast<size_t>(p.C0) * ((p.Cin * 9 + 3) & ~3)) * sizeof(float);
    if (smem > 200 * 1024) return dn_fail(DN_ERR_UNSUPPORTED, "intro: too many channels");
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(intro_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             200 * 1024);
        if (e != cudaSuccess) return dn_cuda_fail(e, "intro: set smem attribute");
        configured = true;
    }
    dim3 grid((p.Wp + kTile - 1) / kTile, (p.Hp + kTile - 1) / kTile, p.N);
    const cudaError_t le = launch_pdl(intro_kernel, grid, dim3(256), smem, s, p);
    if (le != cudaSuccess) return dn_cuda_fail(le, "intro: launch");
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "intro: launch");
}

int launch_ending(const EndingParams& p, cudaStream_t s) {
    if (p.C0 % 8 != 0) return dn_fail(DN_ERR_UNSUPPORTED, "ending: base channels must be a multiple of 8");
    const size_t smem = static_cast<size_t>(27) * p.C0 * sizeof(float) +
                        static_cast<size_t>((kTile + 2) * (kTile + 2)) * (p.C0 + 2) * sizeof(__half);
    if (smem > 200 * 1024) return dn_fail(DN_ERR_UNSUPPORTED, "ending: too many channels");
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(ending_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             200 * 1024);
        if (e != cudaSuccess) return dn_cuda_fail(e, "ending: set smem attribute");
        configured = true;
    }
    dim3 grid((p.W + kTile - 1) / kTile, (p.H + kTile - 1) / kTile, p.N);
    const cudaError_t le = launch_pdl(ending_kernel, grid, dim3(256), smem, s, p);
    if (le != cudaSuccess) return dn_cuda_fail(le, "ending: launch");
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "ending: launch");
}

}  // namespace dnb
