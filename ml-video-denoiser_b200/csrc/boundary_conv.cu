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

constexpr int kTH = 8, kTW = 32;        // output tile; 128 threads, two pixels each
constexpr int kHH = kTH + 2, kWW = kTW + 2;
constexpr int kArea = kHH * kWW;        // halo pixels
constexpr int kThreads = 128;

__device__ __forceinline__ float finite_or_zero(float v) {
    return (isnan(v) || isinf(v)) ? 0.f : v;
}

__device__ __forceinline__ int reflect_hi(int i, int n) { return i < n ? i : 2 * (n - 1) - i; }

// Thread t owns pixels (t / 16, t % 16) and (t / 16, t % 16 + 16) of the
// tile: the lanes of a warp read consecutive halo pixels (conflict-free
// shared-memory reads) and both pixels share every broadcast weight load.

// Intro: one pass per group of NP output-channel pairs (2*NP channels).
// acc pair (o, o+1) of pixel q += (v, v) * (w[k][o], w[k][o+1]) in packed
// fp32 FMAs; weights are broadcast float4 reads of sw[k][C0].
template <int NP>
__device__ __forceinline__ void intro_group(const float* sx, const float* sw, const float* bias, int Cin, int C0,
                                            int o0, int ly, int lx, __half* dst0, __half* dst1, bool st0, bool st1) {
    float2 acc[2][NP];
#pragma unroll
    for (int j = 0; j < NP; ++j) acc[0][j] = acc[1][j] = make_float2(bias[o0 + 2 * j], bias[o0 + 2 * j + 1]);
    for (int c = 0; c < Cin; ++c) {
        const float* xc = sx + c * kArea;
#pragma unroll
        for (int t = 0; t < 9; ++t) {
            const int r = (ly + t / 3) * kWW + lx + t % 3;
            const float v0 = xc[r], v1 = xc[r + 16];
            const float2 a = make_float2(v0, v0), b = make_float2(v1, v1);
            const float4* wr = reinterpret_cast<const float4*>(sw + (c * 9 + t) * C0 + o0);
#pragma unroll
            for (int j = 0; j < NP / 2; ++j) {
                const float4 w4 = wr[j];
                const float2 wa = make_float2(w4.x, w4.y), wb = make_float2(w4.z, w4.w);
                acc[0][2 * j] = ffma2(a, wa, acc[0][2 * j]);
                acc[0][2 * j + 1] = ffma2(a, wb, acc[0][2 * j + 1]);
                acc[1][2 * j] = ffma2(b, wa, acc[1][2 * j]);
                acc[1][2 * j + 1] = ffma2(b, wb, acc[1][2 * j + 1]);
            }
        }
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        if (!(q ? st1 : st0)) continue;
        __half* d = (q ? dst1 : dst0) + o0;
#pragma unroll
        for (int j = 0; j < NP; j += 4) {
            uint4 ov;
            ov.x = pack_half2(acc[q][j].x, acc[q][j].y);
            ov.y = pack_half2(acc[q][j + 1].x, acc[q][j + 1].y);
            ov.z = pack_half2(acc[q][j + 2].x, acc[q][j + 2].y);
            ov.w = pack_half2(acc[q][j + 3].x, acc[q][j + 3].y);
            *reinterpret_cast<uint4*>(d + 2 * j) = ov;
        }
    }
}

__global__ void __launch_bounds__(kThreads) intro_kernel(const __grid_constant__ IntroParams p) {
    extern __shared__ __align__(16) float sm[];
    const int Cin = p.Cin, C0 = p.C0;
    float* sw = sm;                   // [Cin*9][C0]
    float* sb = sw + Cin * 9 * C0;    // [C0]
    float* sx = sb + C0;              // [Cin][kHH][kWW]
    const int img = blockIdx.z;
    const int ty0 = blockIdx.y * kTH, tx0 = blockIdx.x * kTW;
    const __half* x = p.x + static_cast<size_t>(img) * p.in_batch_stride;
    const int tid = threadIdx.x;
    pdl_trigger();
    for (int i = tid; i < Cin * 9 * C0; i += kThreads) {
        const int k = i / C0, o = i - k * C0;
        sw[i] = p.w[o * Cin * 9 + k];
    }
    for (int i = tid; i < C0; i += kThreads) sb[i] = p.b[i];
    pdl_wait();
    // Halo staging in batches of kBatch loads per thread, all issued before
    // any is used (one memory latency per batch).
    constexpr int kBatch = 12;
    for (int base = tid; base < Cin * kArea; base += kBatch * kThreads) {
        __half hv[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const int i = base + j * kThreads;
            hv[j] = __float2half(0.f);  // conv zero padding outside the padded frame
            if (i < Cin * kArea) {
                const int c = i / kArea;
                const int r = i - c * kArea;
                const int yy = ty0 + r / kWW - 1;  // coordinate in the padded frame
                const int xx = tx0 + r % kWW - 1;
                if (yy >= 0 && yy < p.Hp && xx >= 0 && xx < p.Wp)
                    hv[j] = x[(static_cast<size_t>(c) * p.H + reflect_hi(yy, p.H)) * p.W + reflect_hi(xx, p.W)];
            }
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const int i = base + j * kThreads;
            if (i < Cin * kArea) sx[i] = finite_or_zero(__half2float(hv[j]));
        }
    }
    __syncthreads();
    const int ly = tid >> 4, lx = tid & 15;
    const int oy = ty0 + ly, ox0 = tx0 + lx;
    if (oy >= p.Hp) return;
    __half* row = p.y + (static_cast<size_t>(img) * p.Hp + oy) * p.Wp * C0;
    __half* d0 = row + static_cast<size_t>(ox0) * C0;
    __half* d1 = row + static_cast<size_t>(ox0 + 16) * C0;
    const bool st0 = ox0 < p.Wp, st1 = ox0 + 16 < p.Wp;
    int o0 = 0;
    for (; o0 + 16 <= C0; o0 += 16) intro_group<8>(sx, sw, sb, Cin, C0, o0, ly, lx, d0, d1, st0, st1);
    if (o0 < C0) intro_group<4>(sx, sw, sb, Cin, C0, o0, ly, lx, d0, d1, st0, st1);
}

// Ending: output tile 16 x 32; thread = one column x 4 output rows, so per
// tap column kx and 8 channels it loads the 6 halo rows it needs once and
// uses them for all 3 tap rows, and every broadcast weight read serves 4
// pixels. The halo of the NHWC features is staged as fp16 by cp.async (zero
// fill outside the padded map; pixel stride C0 + 8 halves: consecutive lanes
// hit distinct 16-byte bank groups). Packed FMAs accumulate even and odd
// channels in the two lanes.
constexpr int kETH = 16, kETW = 32;
constexpr int kEWW = kETW + 2;
constexpr int kEArea = (kETH + 2) * kEWW;

__global__ void __launch_bounds__(kThreads) ending_kernel(const __grid_constant__ EndingParams p) {
    extern __shared__ __align__(16) float sm[];
    const int C0 = p.C0;
    const int ps = C0 + 8;                                  // halves per staged halo pixel
    float* sw = sm;                                         // [9 taps][C0/8][3 outputs][8]
    __half* sx = reinterpret_cast<__half*>(sw + 27 * C0);   // [kEArea][ps]
    const int img = blockIdx.z;
    const int ty0 = blockIdx.y * kETH, tx0 = blockIdx.x * kETW;
    const int tid = threadIdx.x;
    pdl_trigger();
    for (int i = tid; i < 27 * C0; i += kThreads) {
        const int t = i / (3 * C0);
        const int r = i - t * 3 * C0;
        const int c8 = r / 24, o = (r / 8) % 3, e = r % 8;
        sw[i] = p.w[(o * 9 + t) * C0 + 8 * c8 + e];
    }
    pdl_wait();
    const __half* xin = p.x + static_cast<size_t>(img) * p.Hp * p.Wp * C0;
    const int vec = C0 / 8;
    for (int i = tid; i < kEArea * vec; i += kThreads) {
        const int r = i / vec;
        const int q = i - r * vec;
        const int yy = ty0 + r / kEWW - 1;
        const int xx = tx0 + r % kEWW - 1;
        const bool valid = yy >= 0 && yy < p.Hp && xx >= 0 && xx < p.Wp;
        const __half* src = valid ? xin + (static_cast<size_t>(yy) * p.Wp + xx) * C0 + q * 8 : xin;
        cp_async16_zfill(sx + static_cast<size_t>(r) * ps + q * 8, src, valid);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    const int lx = tid & 31, rg = tid >> 5;  // column, group of 4 output rows
    float2 acc[4][3];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int o = 0; o < 3; ++o) acc[r][o] = make_float2(0.f, 0.f);
#pragma unroll 1
    for (int c8 = 0; c8 < C0 / 8; ++c8) {
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
            float2 in[6][4];  // halo rows 4rg .. 4rg+5 at column lx+kx, channels 8c8 .. 8c8+7
#pragma unroll
            for (int ir = 0; ir < 6; ++ir) {
                const uint4 v = *reinterpret_cast<const uint4*>(
                    sx + static_cast<size_t>((4 * rg + ir) * kEWW + lx + kx) * ps + 8 * c8);
                in[ir][0] = unpack_half2(v.x);
                in[ir][1] = unpack_half2(v.y);
                in[ir][2] = unpack_half2(v.z);
                in[ir][3] = unpack_half2(v.w);
            }
#pragma unroll
            for (int ky = 0; ky < 3; ++ky) {
                const float4* wt = reinterpret_cast<const float4*>(sw + ((ky * 3 + kx) * (C0 / 8) + c8) * 24);
                float2 w[3][4];
#pragma unroll
                for (int o = 0; o < 3; ++o) {
                    const float4 a = wt[2 * o], b = wt[2 * o + 1];
                    w[o][0] = make_float2(a.x, a.y);
                    w[o][1] = make_float2(a.z, a.w);
                    w[o][2] = make_float2(b.x, b.y);
                    w[o][3] = make_float2(b.z, b.w);
                }
#pragma unroll
                for (int orow = 0; orow < 4; ++orow)
#pragma unroll
                    for (int o = 0; o < 3; ++o)
#pragma unroll
                        for (int e = 0; e < 4; ++e) acc[orow][o] = ffma2(in[orow + ky][e], w[o][e], acc[orow][o]);
            }
        }
    }
    const size_t plane = static_cast<size_t>(p.H) * p.W;
    const __half* beauty = p.beauty + static_cast<size_t>(img) * p.beauty_batch_stride;
    __half* out = p.y + static_cast<size_t>(img) * 3 * plane;
    const int ox = tx0 + lx;
    if (ox >= p.W) return;
#pragma unroll
    for (int orow = 0; orow < 4; ++orow) {
        const int oy = ty0 + 4 * rg + orow;
        if (oy >= p.H) break;
        const size_t o = static_cast<size_t>(oy) * p.W + ox;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            const float r = (acc[orow][c].x + acc[orow][c].y) + p.b[c];
            out[c * plane + o] = __float2half(finite_or_zero(__half2float(beauty[c * plane + o])) + r);
        }
    }
}

}  // namespace

int launch_intro(const IntroParams& p, cudaStream_t s) {
    if (p.C0 % 8 != 0) return dn_fail(DN_ERR_UNSUPPORTED, "intro: base channels must be a multiple of 8");
    const size_t smem = (static_cast<size_t>(p.Cin) * kArea + static_cast<size_t>(p.C0) * (p.Cin * 9 + 1)) *
                        sizeof(float);
    if (smem > 200 * 1024) return dn_fail(DN_ERR_UNSUPPORTED, "intro: too many channels");
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(intro_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             200 * 1024);
        if (e != cudaSuccess) return dn_cuda_fail(e, "intro: set smem attribute");
        configured = true;
    }
    dim3 grid((p.Wp + kTW - 1) / kTW, (p.Hp + kTH - 1) / kTH, p.N);
    const cudaError_t le = launch_pdl(intro_kernel, grid, dim3(kThreads), smem, s, p);
    if (le != cudaSuccess) return dn_cuda_fail(le, "intro: launch");
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "intro: launch");
}

int launch_ending(const EndingParams& p, cudaStream_t s) {
    if (p.weff && ending_tc_supported(p.C0)) return launch_ending_tc(p, s);
    if (p.C0 % 8 != 0) return dn_fail(DN_ERR_UNSUPPORTED, "ending: base channels must be a multiple of 8");
    const size_t smem = static_cast<size_t>(27) * p.C0 * sizeof(float) +
                        static_cast<size_t>(kEArea) * (p.C0 + 8) * sizeof(__half);
    if (smem > 200 * 1024) return dn_fail(DN_ERR_UNSUPPORTED, "ending: too many channels");
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(ending_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             200 * 1024);
        if (e != cudaSuccess) return dn_cuda_fail(e, "ending: set smem attribute");
        configured = true;
    }
    dim3 grid((p.W + kETW - 1) / kETW, (p.H + kETH - 1) / kETH, p.N);
    const cudaError_t le = launch_pdl(ending_kernel, grid, dim3(kThreads), smem, s, p);
    if (le != cudaSuccess) return dn_cuda_fail(le, "ending: launch");
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "ending: launch");
}

}  // namespace dnb
