// The intro conv (3x3, Cin -> C0) on the tensor cores as an im2col GEMM:
// for each output pixel the K = 9 * Cin inputs of its 3x3 window (k = c*9 +
// ky*3 + kx, zero-padded to a multiple of 16) form one A row, so a strip
// row of 128 pixels is one M = 128, N = C0 MMA chain of K/16 steps with no
// inflation of the MACs (the window is built in shared memory, not
// multiplied out as shifted copies of the input).
//
// A CTA (128 threads, thread = pixel = TMEM lane) walks the rows of a strip
// segment: per output row it loads one new input row of the strip (130
// pixels of each channel, with the right/bottom reflect pad of the padded
// frame, the conv's zero padding outside it, and nan_to_num), keeps the
// last three in a shared ring, builds the A tile, issues the MMAs, and
// stores the row (+ bias) to the NHWC output. Small CTAs (a 32-column TMEM
// accumulator, ~15-40 KB of shared memory) run many per SM, which is what
// hides the per-row latencies.
//
// Replaces the reference's reflect_pad_kernel and the intro cudnnConvolutionForward
// + bias pass (src/models/nafnet.cu:354-357, src/kernels/model_kernels.cu:15-34),
// with nan_to_num on the input as in training/models.py:559.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "kernels.h"
#include "launch.cuh"
#include "sm100.cuh"
#include "status.h"

namespace dnb {
int sm_count();

namespace {

constexpr int kIT = 128;      // threads = strip pixels = MMA M
constexpr int kHP = kIT + 2;  // input pixels per strip row (halo)

__device__ __forceinline__ float finite0(float v) { return (isnan(v) || isinf(v)) ? 0.f : v; }
__device__ __forceinline__ int reflect_hi(int i, int n) { return i < n ? i : 2 * (n - 1) - i; }

// Shared memory: A tile [KP/8][128 rows][8] fp16 | B [C0 rows][KP] fp16, both
// no-swizzle K-major | input ring [3][Cin][kHP] fp32 | bias [C0].
__host__ __device__ constexpr int intro_smem(int Cin, int C0, int KP) {
    return 128 + kIT * KP * 2 + C0 * KP * 2 + 3 * Cin * kHP * 4 + C0 * 4;
}

// KP = 9 * Cin rounded up to 16 (32 for RGB); kR = input-row elements per
// thread (Cin * kHP / 128, rounded up) for the largest Cin of that KP.
template <int C0, int KP>
__global__ void __launch_bounds__(kIT) intro_tc_kernel(const __grid_constant__ IntroParams p, unsigned strips) {
    constexpr uint32_t kCols = C0 < 32 ? 32 : C0;
    constexpr int kR = ((KP / 9) * kHP + kIT - 1) / kIT;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
    uint8_t* sA = smem;
    uint8_t* sB = sA + kIT * KP * 2;
    float* sIn = reinterpret_cast<float*>(sB + C0 * KP * 2);  // [3][Cin][kHP]
    float* sBias = sIn + 3 * p.Cin * kHP;
    __shared__ uint64_t bar_mma;
    __shared__ uint32_t tslot;

    const int tid = threadIdx.x, warp = tid >> 5;
    const int Cin = p.Cin, K = 9 * Cin, RN = Cin * kHP;
    // Weights -> B (fp16, zero for k >= K), bias.
    for (int i = tid; i < C0 * KP; i += kIT) {
        const int o = i / KP, k = i - o * KP;
        const float v = k < K ? p.w[o * K + k] : 0.f;
        *reinterpret_cast<__half*>(sB + kmajor_offset(o, k >> 3, (KP / 8) * 128) + (k & 7) * 2) = __float2half(v);
    }
    for (int i = tid; i < C0; i += kIT) sBias[i] = p.b[i];
    if (warp == 0) {
        tmem_alloc(&tslot, kCols);
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(&bar_mma, 1);
        fence_mbar_init();
    }
    fence_async_smem();  // B was written by the generic proxy
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    pdl_trigger();  // only once this CTA holds its TMEM columns
    pdl_wait();     // the input may come from the previous kernel

    const int Hp = p.Hp, Wp = p.Wp;
    const long long per_img = static_cast<long long>(strips) * Hp;
    const long long T = per_img * p.N;
    const long long u1 = T * (blockIdx.x + 1) / gridDim.x;
    long long u = T * blockIdx.x / gridDim.x;
    const uint64_t da = sdesc_kmajor(smem_u32(sA), kIT * 16, 128);
    const uint64_t db = sdesc_kmajor(smem_u32(sB), 128, (KP / 8) * 128);
    constexpr uint32_t idesc = idesc_f16_f32(128, C0);
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    uint32_t phase = 0;
    bool ok = true;
    while (ok && u < u1) {
        const int img = static_cast<int>(u / per_img);
        const long long rem = u - img * per_img;
        const int strip = static_cast<int>(rem / Hp);
        const int ya = static_cast<int>(rem - static_cast<long long>(strip) * Hp);
        const int yb = static_cast<int>(std::min<long long>(Hp - 1, ya + (u1 - u) - 1));
        const int x0 = strip * kIT;
        const __half* xin = p.x + static_cast<size_t>(img) * p.in_batch_stride;
        // Row yy of the padded frame (the conv's zero padding outside it;
        // right/bottom reflect inside), element i = c * kHP + j of the strip.
        auto fetch = [&](int yy, float (&r)[kR]) {
#pragma unroll
            for (int q = 0; q < kR; ++q) {
                const int i = tid + q * kIT;
                const int c = i / kHP, xx = x0 - 1 + (i - c * kHP);
                float v = 0.f;
                if (i < RN && yy >= 0 && yy < Hp && xx >= 0 && xx < Wp)
                    v = finite0(__half2float(
                        xin[(static_cast<size_t>(c) * p.H + reflect_hi(yy, p.H)) * p.W + reflect_hi(xx, p.W)]));
                r[q] = v;
            }
        };
        auto put = [&](int yy, const float (&r)[kR]) {
            float* dst = sIn + ((yy + 3) % 3) * RN;
#pragma unroll
            for (int q = 0; q < kR; ++q)
                if (tid + q * kIT < RN) dst[tid + q * kIT] = r[q];
        };
        float nxt[kR];
        fetch(ya - 1, nxt);
        put(ya - 1, nxt);
        fetch(ya, nxt);
        put(ya, nxt);
        fetch(ya + 1, nxt);
        for (int y = ya; y <= yb; ++y) {
            put(y + 1, nxt);
            __syncthreads();  // the three rows are in place
            // A row of pixel tid: k = c*9 + ky*3 + kx.
            const float* rows[3] = {sIn + ((y + 2) % 3) * RN + tid, sIn + (y % 3) * RN + tid,
                                    sIn + ((y + 1) % 3) * RN + tid};
#pragma unroll
            for (int kg = 0; kg < KP / 8; ++kg) {
                float f[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int k = kg * 8 + i;
                    const int c = k / 9, ky = (k % 9) / 3, kx = k % 3;
                    f[i] = k < K ? rows[ky][c * kHP + kx] : 0.f;
                }
                *reinterpret_cast<uint4*>(sA + kg * (kIT * 16) + tid * 16) = f_to_h8(f);
            }
            fence_async_smem();
            tc_fence_before();
            __syncthreads();
            if (tid == 0) {
                tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < KP / 16; ++ks)
                    mma_f16(tmem, desc_add(da, ks * 2 * kIT * 16), desc_add(db, ks * 256), idesc, ks > 0 ? 1u : 0u);
                mma_commit(&bar_mma);
            }
            if (y < yb) fetch(y + 2, nxt);  // in flight while the MMA runs
            const bool got = mbar_wait(&bar_mma, phase);
            if (!__syncthreads_and(got)) {  // every thread leaves together
                if (tid == 0) report_error(p.err, 0xb0, kErrMbarTimeout);
                ok = false;
                break;
            }
            phase ^= 1u;
            tc_fence_after();
            const int ox = x0 + tid;
            __half* dst = p.y + ((static_cast<size_t>(img) * Hp + y) * Wp + ox) * C0;
#pragma unroll
            for (int c0 = 0; c0 < C0; c0 += 16) {
                float v[16];
                tmem_ld16(lane_base + c0, v);
                tmem_ld_wait();
                if (ox < Wp) {
#pragma unroll
                    for (int h = 0; h < 16; h += 8) {
                        float f[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) f[i] = v[h + i] + sBias[c0 + h + i];
                        *reinterpret_cast<uint4*>(dst + c0 + h) = f_to_h8(f);
                    }
                }
            }
            tc_fence_before();  // the next row's MMA overwrites the accumulator
        }
        u += yb - ya + 1;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, kCols);
}

template <int C0, int KP>
int run_intro_tc(const IntroParams& p, cudaStream_t s) {
    constexpr int kMaxSmem = intro_smem(KP / 9, C0, KP);
    static bool configured = false;
    if (!configured) {
        cudaError_t e =
            cudaFuncSetAttribute(intro_tc_kernel<C0, KP>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
        if (e != cudaSuccess) return dn_cuda_fail(e, "intro_tc: smem attribute");
        configured = true;
    }
    const int smem = intro_smem(p.Cin, C0, KP);
    const unsigned strips = static_cast<unsigned>((p.Wp + kIT - 1) / kIT);
    const long long units = static_cast<long long>(strips) * p.Hp * p.N;
    // Up to 8 CTAs per SM (8 x 32 TMEM columns at C0 <= 32; the row latencies
    // of one CTA overlap those of the others), at least ~8 rows per CTA.
    const long long grid = std::max(1LL, std::min<long long>((units + 7) / 8, static_cast<long long>(sm_count()) * 8));
    cudaError_t e = launch_pdl(intro_tc_kernel<C0, KP>, dim3(static_cast<unsigned>(grid)), dim3(kIT), smem, s, p, strips);
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "intro_tc: launch");
}

template <int C0>
int run_intro_tc_k(const IntroParams& p, cudaStream_t s) {
    if (p.Cin <= 3) return run_intro_tc<C0, 32>(p, s);
    if (p.Cin <= 7) return run_intro_tc<C0, 64>(p, s);
    return run_intro_tc<C0, 128>(p, s);
}

}  // namespace

bool intro_tc_supported(int Cin, int C0) { return Cin >= 1 && Cin <= 14 && (C0 == 16 || C0 == 32 || C0 == 64); }

int launch_intro_tc(const IntroParams& p, cudaStream_t s) {
    if (!intro_tc_supported(p.Cin, p.C0)) return dn_fail(DN_ERR_UNSUPPORTED, "intro_tc: channel configuration");
    if (reinterpret_cast<uintptr_t>(p.y) & 15) return dn_fail(DN_ERR_INVALID_ARG, "intro_tc: y must be 16-byte aligned");
    if (p.C0 == 16) return run_intro_tc_k<16>(p, s);
    if (p.C0 == 32) return run_intro_tc_k<32>(p, s);
    return run_intro_tc_k<64>(p, s);
}

}  // namespace dnb
