// Row-panel implicit GEMM on the 5th-generation tensor cores (tcgen05).
//
// One CTA (4 warps) owns a 128-row x NT-column output tile. Thread t owns
// row t end to end: it gathers its A row (1x1 pixel rows, 2x2/stride-2
// patches, or a channel concat of up to 8 sources), applies the fused
// prologue (LayerNorm over K, or the SCA channel scale), writes the row into
// the no-swizzle K-major operand layout, and after the MMA reads its row of
// the fp32 accumulator back from TMEM lane t for the fused epilogue (bias,
// SimpleGate, beta/gamma residual, or PixelShuffle(2) scatter + skip add).
//
// K runs in chunks of KC (<= 64) through a 2-stage pipeline: B tiles are
// pre-packed on the host in the exact shared-memory image and arrive by one
// TMA bulk copy per chunk (mbarrier complete_tx); A tiles are produced by the
// threads; one elected thread issues KC/16 tcgen05.mma (M=128, N=NT, K=16)
// per chunk and commits them to the stage's mbarrier, which both frees the
// stage for reuse and, for the last chunk, releases the epilogue.
//
// Replaces the reference's cudnnConvolutionForward + cudnnAddTensor pair
// (src/layers/conv2d.cu:94-150) and the separate LN / SimpleGate / SCA /
// scaled-add / pixel-shuffle / add kernels (src/kernels/nafnet_kernels.cu
// :54-208) that surround each 1x1 / 2x2 conv of a NAFBlock
// (src/models/nafnet.cu:146-255).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kernels.h"
#include "sm100.cuh"
#include "status.h"

namespace dnb {
namespace {

constexpr int kRows = 128;

__device__ __forceinline__ void h8_to_f(const uint4& v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = unpack_half2(w[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

__device__ __forceinline__ uint4 f_to_h8(const float (&f)[8]) {
    uint4 v;
    v.x = pack_half2(f[0], f[1]);
    v.y = pack_half2(f[2], f[3]);
    v.z = pack_half2(f[4], f[5]);
    v.w = pack_half2(f[6], f[7]);
    return v;
}

// Source address of the 8 channels [k, k+8) of the A row at (img, pix) of
// the GEMM row grid.
template <int AMODE>
__device__ __forceinline__ const __half* a_src(const GemmParams& p, int img, int pix, int k) {
    const int seg = k / p.seg_c;
    const int c = k - seg * p.seg_c;
    if (AMODE == kARows) {
        return p.a[seg] + img * p.a_img_stride + static_cast<size_t>(pix) * p.seg_c + c;
    } else {
        // seg = tap (ky*2 + kx) of the 2x2 stride-2 patch
        const int y = pix / p.Wo;
        const int x = pix - y * p.Wo;
        const size_t spix = static_cast<size_t>(2 * y + (seg >> 1)) * (2 * p.Wo) + 2 * x + (seg & 1);
        return p.a[0] + img * p.a_img_stride + spix * p.seg_c + c;
    }
}

template <int PRO, int EPI, int AMODE, int NT>
__global__ void __launch_bounds__(128) gemm_tc_kernel(const __grid_constant__ GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ uint64_t bar_mma[2];
    __shared__ uint64_t bar_b[2];
    __shared__ uint32_t tslot;
    __shared__ int s_fail;

    constexpr uint32_t kCols = NT < 32 ? 32 : NT;
    const int KC = p.KC;
    const uint32_t a_bytes = kRows * KC * 2;
    const uint32_t b_bytes = NT * KC * 2;
    const uint32_t sbo = static_cast<uint32_t>(KC / 8) * 128u;
    uint8_t* sA0 = smem;
    uint8_t* sB0 = smem + 2 * a_bytes;

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int n_tile = blockIdx.x % p.n_tiles;
    const int m_tile = blockIdx.x / p.n_tiles;
    const int row = m_tile * kRows + tid;
    const bool row_ok = row < p.M;
    const int img = row_ok ? row / p.hw : 0;
    const int pix = row - img * p.hw;

    if (warp == 0) {
        tmem_alloc(&tslot, kCols);
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(&bar_mma[0], 1);
        mbar_init(&bar_mma[1], 1);
        mbar_init(&bar_b[0], 1);
        mbar_init(&bar_b[1], 1);
        s_fail = 0;
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;

    // LayerNorm statistics of this row (two passes over K; the row is
    // re-read from L1/L2 by the chunk loop below).
    float mean = 0.f, rstd = 0.f;
    if (PRO == kProLayerNorm && row_ok) {
        float s = 0.f;
        for (int k = 0; k < p.K; k += 8) {
            float f[8];
            h8_to_f(__ldg(reinterpret_cast<const uint4*>(a_src<AMODE>(p, img, pix, k))), f);
#pragma unroll
            for (int i = 0; i < 8; ++i) s += f[i];
        }
        mean = s / static_cast<float>(p.K);
        float v = 0.f;
        for (int k = 0; k < p.K; k += 8) {
            float f[8];
            h8_to_f(__ldg(reinterpret_cast<const uint4*>(a_src<AMODE>(p, img, pix, k))), f);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float d = f[i] - mean;
                v += d * d;
            }
        }
        rstd = rsqrtf(v / static_cast<float>(p.K) + 1e-6f);
    }

    const int nk = p.k_chunks;
    const uint32_t idesc = idesc_f16_f32(kRows, NT);
    bool ok = true;
    for (int j = 0; j < nk; ++j) {
        const int buf = j & 1;
        uint8_t* sA = sA0 + buf * a_bytes;
        uint8_t* sB = sB0 + buf * b_bytes;
        if (j >= 2) {
            // The MMAs of chunk j-2 must be done reading this stage.
            const bool w = mbar_wait(&bar_mma[buf], ((j - 2) >> 1) & 1);
            if (!w) report_error(p.err, 0x10, kErrMbarTimeout);
            ok = __syncthreads_and(w) != 0;
            if (!ok) break;
        }
        if (tid == 0) {
            mbar_arrive_expect_tx(&bar_b[buf], b_bytes);
            bulk_g2s(sB, p.bpack + (static_cast<size_t>(n_tile) * nk + j) * b_bytes, b_bytes,
                     &bar_b[buf]);
        }
        // A chunk: this thread's row, KC/8 vectors of 8 channels.
        const int k0 = j * KC;
        uint4 v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int k = k0 + q * 8;
            v[q] = make_uint4(0, 0, 0, 0);
            if (q * 8 < KC && row_ok && k < p.K)
                v[q] = __ldg(reinterpret_cast<const uint4*>(a_src<AMODE>(p, img, pix, k)));
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            if (q * 8 >= KC) break;
            const int k = k0 + q * 8;
            if (PRO != kProNone && row_ok && k < p.K) {
                float f[8];
                h8_to_f(v[q], f);
                if (PRO == kProLayerNorm) {
                    const float4 w0 = __ldg(reinterpret_cast<const float4*>(p.pro_w + k));
                    const float4 w1 = __ldg(reinterpret_cast<const float4*>(p.pro_w + k + 4));
                    const float4 b0 = __ldg(reinterpret_cast<const float4*>(p.pro_b + k));
                    const float4 b1 = __ldg(reinterpret_cast<const float4*>(p.pro_b + k + 4));
                    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                    const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                    for (int i = 0; i < 8; ++i) f[i] = (f[i] - mean) * rstd * wv[i] + bv[i];
                } else {
                    const float* sc = p.pro_scale + static_cast<size_t>(img) * p.K + k;
                    const float4 s0 = __ldg(reinterpret_cast<const float4*>(sc));
                    const float4 s1 = __ldg(reinterpret_cast<const float4*>(sc + 4));
                    const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
                    for (int i = 0; i < 8; ++i) f[i] *= sv[i];
                }
                v[q] = f_to_h8(f);
            }
            *reinterpret_cast<uint4*>(sA + kmajor_offset(tid, q, sbo)) = v[q];
        }
        fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            if (!mbar_wait(&bar_b[buf], (j >> 1) & 1)) {
                report_error(p.err, 0x11, kErrMbarTimeout);
                s_fail = 1;
            } else {
                tc_fence_after();
                const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
                for (int s = 0; s < KC / 16; ++s) {
                    mma_f16(tmem, sdesc_kmajor(a0 + s * 256, 128, sbo),
                            sdesc_kmajor(b0 + s * 256, 128, sbo), idesc,
                            (j > 0 || s > 0) ? 1u : 0u);
                }
            }
            mma_commit(&bar_mma[buf]);
        }
    }

    if (ok) {
        const bool w = mbar_wait(&bar_mma[(nk - 1) & 1], ((nk - 1) >> 1) & 1);
        if (!w) report_error(p.err, 0x12, kErrMbarTimeout);
        ok = __syncthreads_and(w && s_fail == 0) != 0;
    }
    tc_fence_after();

    if (ok) {
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
        if (EPI == kEpiGate) {
            constexpr int kHalf = NT / 2;
#pragma unroll 1
            for (int c0 = 0; c0 < kHalf; c0 += 16) {
                float va[16], vb[16];
                tmem_ld16(lane_base + c0, va);
                tmem_ld16(lane_base + kHalf + c0, vb);
                tmem_ld_wait();
                const int o0 = n_tile * kHalf + c0;
                if (!row_ok || o0 >= p.n_out) continue;
                const float* bias = p.bias + n_tile * NT;
                float r[16];
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    r[i] = (va[i] + bias[c0 + i]) * (vb[i] + bias[kHalf + c0 + i]);
                __half* dst = p.out + static_cast<size_t>(row) * p.out_c + o0;
#pragma unroll
                for (int g = 0; g < 2; ++g) {
                    if (o0 + 8 * g >= p.n_out) break;
                    float f[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) f[i] = r[8 * g + i];
                    *reinterpret_cast<uint4*>(dst + 8 * g) = f_to_h8(f);
                }
            }
        } else {
#pragma unroll 1
            for (int c0 = 0; c0 < NT; c0 += 16) {
                float va[16];
                tmem_ld16(lane_base + c0, va);
                tmem_ld_wait();
                const int n0 = n_tile * NT + c0;
                if (!row_ok || n0 >= p.n_out) continue;
#pragma unroll
                for (int g = 0; g < 2; ++g) {
                    const int n = n0 + 8 * g;
                    if (n >= p.n_out) break;
                    float f[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        f[i] = va[8 * g + i] + (p.bias ? p.bias[n + i] : 0.f);
                    if (EPI == kEpiStore) {
                        *reinterpret_cast<uint4*>(p.out + static_cast<size_t>(row) * p.out_c + n) =
                            f_to_h8(f);
                    } else if (EPI == kEpiResidual) {
                        const size_t off = static_cast<size_t>(row) * p.out_c + n;
                        float r[8];
                        h8_to_f(*reinterpret_cast<const uint4*>(p.res + off), r);
#pragma unroll
                        for (int i = 0; i < 8; ++i) f[i] = r[i] + p.res_scale[n + i] * f[i];
                        *reinterpret_cast<uint4*>(p.out + off) = f_to_h8(f);
                    } else {  // kEpiShuffleAdd: column n -> (sub-pixel ij, channel ch)
                        const int cout = p.out_c;
                        const int ij = n / cout;
                        const int ch = n - ij * cout;
                        const int y = pix / p.Wo;
                        const int x = pix - y * p.Wo;
                        const size_t pix =
                            (static_cast<size_t>(img) * (2 * p.Ho) + 2 * y + (ij >> 1)) *
                                (2 * p.Wo) +
                            2 * x + (ij & 1);
                        const size_t off = pix * cout + ch;
                        float r[8];
                        h8_to_f(*reinterpret_cast<const uint4*>(p.skip + off), r);
#pragma unroll
                        for (int i = 0; i < 8; ++i) f[i] += r[i];
                        *reinterpret_cast<uint4*>(p.out + off) = f_to_h8(f);
                    }
                }
            }
        }
    } else {
        // Give in-flight MMAs a bounded chance to drain before TMEM is freed.
        if (tid == 0) {
            mbar_wait(&bar_mma[0], 0, 10000000ull);
            mbar_wait(&bar_mma[1], 0, 10000000ull);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, kCols);
}

template <int PRO, int EPI, int AMODE, int NT>
int launch_one(const GemmParams& p, cudaStream_t s) {
    auto kern = gemm_tc_kernel<PRO, EPI, AMODE, NT>;
    // Always reserve the KC=64 footprint: it caps residency at <= 512 TMEM
    // columns per SM for every NT, so tcgen05.alloc never has to wait.
    const int smem = 2 * (kRows * 64 * 2 + NT * 64 * 2);
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             smem);
        if (e != cudaSuccess) return dn_cuda_fail(e, "gemm: set smem attribute");
        configured = true;
    }
    const int m_tiles = (p.M + kRows - 1) / kRows;
    const long long grid = static_cast<long long>(m_tiles) * p.n_tiles;
    if (grid <= 0 || grid > 0x7fffffffLL) return dn_fail(DN_ERR_INVALID_ARG, "gemm: bad grid");
    kern<<<static_cast<unsigned>(grid), 128, smem, s>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return dn_cuda_fail(e, "gemm: launch");
    return DN_OK;
}

template <int PRO, int EPI, int AMODE>
int launch_nt(const GemmParams& p, int nt, cudaStream_t s) {
    switch (nt) {
        case 16:
            if (EPI == kEpiGate) break;
            return launch_one<PRO, EPI, AMODE, 16>(p, s);
        case 32: return launch_one<PRO, EPI, AMODE, 32>(p, s);
        case 64: return launch_one<PRO, EPI, AMODE, 64>(p, s);
        case 128: return launch_one<PRO, EPI, AMODE, 128>(p, s);
        case 256: return launch_one<PRO, EPI, AMODE, 256>(p, s);
        default: break;
    }
    return dn_fail(DN_ERR_UNSUPPORTED, "gemm: unsupported tile width");
}

}  // namespace

int launch_gemm(const GemmParams& p, int pro, int epi, int amode, int nt, cudaStream_t s) {
    if (p.KC != 16 && p.KC != 32 && p.KC != 48 && p.KC != 64)
        return dn_fail(DN_ERR_UNSUPPORTED, "gemm: KC must be 16/32/48/64");
    if (p.seg_c % 8 != 0) return dn_fail(DN_ERR_UNSUPPORTED, "gemm: channels must be a multiple of 8");
    if (p.M <= 0) return DN_OK;
    if (epi == kEpiGate && !p.bias) return dn_fail(DN_ERR_INVALID_ARG, "gemm: gate epilogue needs a bias");
    // Instantiated combinations (the ones the planner emits).
    if (amode == kARows && pro == kProLayerNorm && epi == kEpiStore)
        return launch_nt<kProLayerNorm, kEpiStore, kARows>(p, nt, s);
    if (amode == kARows && pro == kProLayerNorm && epi == kEpiGate)
        return launch_nt<kProLayerNorm, kEpiGate, kARows>(p, nt, s);
    if (amode == kARows && pro == kProScale && epi == kEpiResidual)
        return launch_nt<kProScale, kEpiResidual, kARows>(p, nt, s);
    if (amode == kARows && pro == kProNone && epi == kEpiResidual)
        return launch_nt<kProNone, kEpiResidual, kARows>(p, nt, s);
    if (amode == kARows && pro == kProNone && epi == kEpiStore)
        return launch_nt<kProNone, kEpiStore, kARows>(p, nt, s);
    if (amode == kARows && pro == kProNone && epi == kEpiShuffleAdd)
        return launch_nt<kProNone, kEpiShuffleAdd, kARows>(p, nt, s);
    if (amode == kAS2x2 && pro == kProNone && epi == kEpiStore)
        return launch_nt<kProNone, kEpiStore, kAS2x2>(p, nt, s);
    return dn_fail(DN_ERR_UNSUPPORTED, "gemm: unsupported prologue/epilogue combination");
}

}  // namespace dnb
