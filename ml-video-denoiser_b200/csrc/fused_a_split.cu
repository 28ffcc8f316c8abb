// Phase A of a 32/64-channel NAFBlock with conv1 on the tensor cores and the
// depthwise 3x3 on the CUDA cores (single image):
//   n  = LayerNorm1(x) without its affine (FP16, as the engine's other LN paths)
//   u  = n (W1 diag(gamma1))^T + b1',  b1' = b1 + W1 beta1      (conv1, 2C outputs)
//   u  = 0 outside the image                                      (the depthwise zero padding)
//   g  = SimpleGate(dw3x3(u) + b_dw)                              (C outputs)
// plus the per-CTA pool partials of g and, in the last CTA, the SCA with its
// scale folded into conv3's weights (sca_fold.cuh).
//
// A CTA walks strips of 126 output columns row by row. Input row r of a
// strip is the 128 pixels [x0 - 1, x0 + 127): exactly one M = 128 MMA, so
// conv1 runs once per input pixel (the halo columns included) with no
// inflation of its MACs, unlike the composed 3x3 form of fused_a_tc.cu
// (9 x conv1's MACs on the tensor cores). Roles:
//   warp 0       producer: the row's pixels (contiguous in NHWC) by one bulk
//                copy into a ring of input-row slots;
//   warps 1-4    LayerNorm of the row in place into the no-swizzle K-major
//                MMA layout [C/8][128][8] (zero outside the image);
//   warp 5       MMA issuer: C/16 MMAs (M = 128, N = 2C, K = 16) per row into
//                a ring of TMEM accumulators;
//   warps 6-9    conv1 epilogue (thread = pixel = TMEM lane): + b1', zero
//                outside the image, FP16 u row into a ring of u rows in shared
//                memory (pixel-major, each pixel padded by 16 bytes so that
//                the 16-byte stores of consecutive pixels hit distinct banks);
//   warps 10-17  depthwise + gate: lane = a pair of gated channels (both gate
//                halves), each warp a run of output columns; a lane keeps the
//                3 x 3 window of its four u channels in registers and reads one
//                new u column (three rows, two halves: 4-byte words, a warp
//                reads whole 64/128-byte channel runs of one pixel, conflict
//                free) per output pixel, 18 packed FP32 FMAs, the gate
//                product, a coalesced g store, and the pool sum of the
//                stored FP16 values.
// Output row y needs u rows y-1, y, y+1: the u ring of four rows lets conv1's
// epilogue run one row ahead of the depthwise warps.
//
// Replaces the reference's layer_norm_affine_kernel, conv1 and the grouped
// conv2 cudnnConvolutionForward calls and simple_gate_kernel
// (src/models/nafnet.cu:146-172, src/kernels/nafnet_kernels.cu:54-106) plus
// the pool's partial sums.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "fused_block.h"
#include "kernels.h"
#include "launch.cuh"
#include "sca_fold.cuh"
#include "sm100.cuh"
#include "status.h"

namespace dnb {
namespace {

constexpr int kSpThreads = 576;  // 18 warps
constexpr int kDwWarps = 8;      // warps 10-17
constexpr int kDw0 = 10;

template <int C>
struct SplitGeo {
    static constexpr int U = 2 * C;               // conv1 outputs (both gate halves)
    static constexpr int D = C;                   // gated channels
    static constexpr int SW = 128;                // input pixels per strip row (= MMA M)
    static constexpr int OW = SW - 2;             // output columns per strip row
    static constexpr int KG = C / 8;              // 16-byte channel groups per pixel
    static constexpr int KGB = SW * 16;           // bytes of one channel group of a row (K-adjacent core matrices)
    static constexpr int ROWB = KG * KGB;         // one input-row slot
    static constexpr int XR = C >= 64 ? 3 : 8;    // input-row slots
    static constexpr int TR = 4;                  // TMEM accumulator slots of U columns
    static constexpr int UR = 4;                  // u-row slots
    static constexpr int UPX = 2 * U + 16;        // bytes per pixel of a u row (16 bytes of padding)
    static constexpr int UROWB = SW * UPX;
    static constexpr int WB = U * C * 2;          // conv1 B tile (one K chunk of C)
    static constexpr int TMEM_COLS = TR * U;
    static constexpr int PAIRS = D / 2;           // gated channel pairs = DW lanes per pixel
    static constexpr int GROUPS = 32 / PAIRS;     // pixel walkers per DW warp
    static constexpr int WALKERS = kDwWarps * GROUPS;
    static constexpr int F_FLOATS = 9 * U + U + U + kDwWarps * D;
    static constexpr int SMEM = 1024 + XR * ROWB + UR * UROWB + WB + F_FLOATS * 4;
    static_assert(TMEM_COLS <= 512, "TMEM ring");
    static_assert(SMEM <= 227 * 1024, "shared memory");
    static_assert(UR * UROWB >= 18 * D * 4, "the SCA scratch reuses the u ring");
};

struct Seg {
    int strip, ya, yb;
};

// Units enumerate (strip, output row) with rows fastest; a segment is the
// run of rows of one strip inside [u, u1).
__device__ __forceinline__ bool seg_at(long long u, long long u1, int H, Seg& s) {
    if (u >= u1) return false;
    s.strip = static_cast<int>(u / H);
    s.ya = static_cast<int>(u - static_cast<long long>(s.strip) * H);
    s.yb = static_cast<int>(min(static_cast<long long>(H - 1), s.ya + (u1 - u) - 1));
    return true;
}

template <int C>
__global__ void __launch_bounds__(kSpThreads, 1) split_a_kernel(const __grid_constant__ FusedAParams p) {
    using G = SplitGeo<C>;
    constexpr int U = G::U, D = G::D;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sX = smem;                                   // XR input-row slots
    uint8_t* sU = sX + G::XR * G::ROWB;                   // UR u rows
    uint8_t* sW = sU + G::UR * G::UROWB;                  // conv1 B tile
    float* sTap = reinterpret_cast<float*>(sW + G::WB);   // [9][U]
    float* sDwB = sTap + 9 * U;                           // [U]
    float* sB1 = sDwB + U;                                // [U]
    float* sPool = sB1 + U;                               // [kDwWarps][D]
    __shared__ uint64_t xfull[G::XR], xready[G::XR], xfree[G::XR];
    __shared__ uint64_t afull[G::TR], aempty[G::TR], ufull[G::UR], ufree[G::UR];
    __shared__ uint64_t bar_w, bar_end;
    __shared__ uint32_t tslot;
    __shared__ volatile int s_abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int H = p.H, W = p.W;
    const int strips = (W + G::OW - 1) / G::OW;
    const long long T = static_cast<long long>(strips) * H;
    const long long u0 = T * blockIdx.x / gridDim.x, u1 = T * (blockIdx.x + 1) / gridDim.x;

    for (int i = tid; i < 9 * U; i += kSpThreads) sTap[i] = p.dw_w[i];
    for (int i = tid; i < U; i += kSpThreads) {
        sDwB[i] = p.dw_b[i];
        sB1[i] = p.c2[i];
    }
    for (int i = tid; i < kDwWarps * D; i += kSpThreads) sPool[i] = 0.f;
    if (warp == 0) {
        tmem_alloc(&tslot, G::TMEM_COLS);
        tmem_relinquish();
    }
    if (tid == 32) {
        for (int s = 0; s < G::XR; ++s) {
            mbar_init(&xfull[s], 1);
            mbar_init(&xready[s], 4);
            mbar_init(&xfree[s], 1);
        }
        for (int t = 0; t < G::TR; ++t) {
            mbar_init(&afull[t], 1);
            mbar_init(&aempty[t], 4);
        }
        for (int s = 0; s < G::UR; ++s) {
            mbar_init(&ufull[s], 4);
            mbar_init(&ufree[s], kDwWarps);
        }
        mbar_init(&bar_w, 1);
        mbar_init(&bar_end, 1);
        s_abort = 0;
        fence_mbar_init();
        mbar_arrive_expect_tx(&bar_w, G::WB);
        bulk_g2s(sW, p.w1, G::WB, &bar_w);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    pdl_trigger();  // only once this CTA holds its TMEM columns
    pdl_wait();     // x was written by the previous kernel; g and the partials are read by it

    Seg sg;
    if (warp == 0) {
        // ------------------------------ producer -----------------------------
        if (lane == 0) {
            uint32_t e = 0;
            for (long long u = u0; !s_abort && seg_at(u, u1, H, sg); u += sg.yb - sg.ya + 1) {
                const int x0 = sg.strip * G::OW;
                for (int r = sg.ya - 1; r <= sg.yb + 1; ++r, ++e) {
                    const uint32_t s = e % G::XR, ph = (e / G::XR) & 1u;
                    if (!wait_or_abort(&xfree[s], ph ^ 1u, &s_abort, p.err, 0xa0)) break;
                    if (r < 0 || r >= H) {
                        mbar_arrive(&xfull[s]);  // zeroed by the LayerNorm warps
                    } else {
                        const int pa = max(0, x0 - 1), pb = min(W, x0 - 1 + G::SW);
                        const uint32_t bytes = static_cast<uint32_t>(pb - pa) * C * 2;
                        mbar_arrive_expect_tx(&xfull[s], bytes);
                        bulk_g2s(sX + s * G::ROWB + (pa - (x0 - 1)) * C * 2,
                                 p.x + (static_cast<size_t>(r) * W + pa) * C, bytes, &xfull[s]);
                    }
                }
            }
            if (s_abort) {
                for (uint32_t k = e > G::XR ? e - G::XR : 0; k < e; ++k)
                    mbar_wait(&xfull[k % G::XR], (k / G::XR) & 1u, 5000000ull);
            }
        }
    } else if (warp <= 4) {
        // ------------------------------ LayerNorm ----------------------------
        // A pixel's C/8 16-byte chunks sit in adjacent lanes; statistics are
        // shifted sums (shift = the pixel's first channel) reduced over them.
        // The row stays in registers until all 128 threads have read the
        // slot, then is written back in the MMA layout [C/8][128][8 ch].
        constexpr int CPX = C / 8, PPR = 128 / CPX, NR = G::SW / PPR;
        const int t = tid - 32;
        const int cq = t % CPX, pl = t / CPX;
        const int lead = lane & ~(CPX - 1);
        uint32_t e = 0;
        bool ok = true;
        for (long long u = u0; ok && seg_at(u, u1, H, sg); u += sg.yb - sg.ya + 1) {
            const int x0 = sg.strip * G::OW;
            for (int r = sg.ya - 1; r <= sg.yb + 1; ++r, ++e) {
                const uint32_t s = e % G::XR, ph = (e / G::XR) & 1u;
                const bool got = wait_or_abort(&xfull[s], ph, &s_abort, p.err, 0xa1);
                if (named_sync_or(1, 128, !got)) {
                    ok = false;
                    break;
                }
                uint8_t* row = sX + s * G::ROWB;
                const bool row_in = r >= 0 && r < H;
                uint4 nv[NR];
#pragma unroll
                for (int k = 0; k < NR; ++k) {
                    const int i = k * PPR + pl;
                    const int xin = x0 - 1 + i;
                    const bool valid = row_in && xin >= 0 && xin < W;
                    const uint4 v = valid ? *reinterpret_cast<const uint4*>(row + i * C * 2 + cq * 16)
                                          : make_uint4(0u, 0u, 0u, 0u);
                    const float xs = __shfl_sync(0xffffffffu, unpack_half2(v.x).x, lead);
                    const float2 nx = make_float2(-xs, -xs), one = make_float2(1.f, 1.f);
                    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
                    float2 a1 = make_float2(0.f, 0.f), a2 = make_float2(0.f, 0.f);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 d = ffma2(unpack_half2(w[j]), one, nx);
                        a1 = ffma2(d, one, a1);
                        a2 = ffma2(d, d, a2);
                    }
                    float s1 = a1.x + a1.y, s2 = a2.x + a2.y;
#pragma unroll
                    for (int m = 1; m < CPX; m <<= 1) {
                        s1 += __shfl_xor_sync(0xffffffffu, s1, m);
                        s2 += __shfl_xor_sync(0xffffffffu, s2, m);
                    }
                    const float dm = s1 * (1.0f / C);
                    const float var = fmaxf(s2 * (1.0f / C) - dm * dm, 0.f);
                    const float rstd = rsqrtf(var + 1e-6f);
                    const float2 rs2 = make_float2(rstd, rstd);
                    const float2 sh2 = make_float2(-(xs + dm) * rstd, -(xs + dm) * rstd);
                    uint32_t o[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 y = ffma2(unpack_half2(w[j]), rs2, sh2);
                        o[j] = pack_half2(y.x, y.y);
                    }
                    nv[k] = valid ? make_uint4(o[0], o[1], o[2], o[3]) : make_uint4(0u, 0u, 0u, 0u);
                }
                named_sync(1, 128);  // every thread has read the pixel-major row
#pragma unroll
                for (int k = 0; k < NR; ++k) {
                    const int i = k * PPR + pl;
                    *reinterpret_cast<uint4*>(row + cq * G::KGB + i * 16) = nv[k];
                }
                fence_async_smem();  // the tensor core reads the row (async proxy)
                __syncwarp();
                if (lane == 0) mbar_arrive(&xready[s]);
            }
        }
    } else if (warp == 5) {
        // ------------------------------ MMA issuer ---------------------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(128, U);
            const uint64_t da = sdesc_kmajor(smem_u32(sX), G::KGB, 128);
            const uint64_t db = sdesc_kmajor(smem_u32(sW), 128, (C / 8) * 128);
            bool ok = wait_or_abort(&bar_w, 0, &s_abort, p.err, 0xa2);
            uint32_t e = 0;
            for (long long u = u0; ok && seg_at(u, u1, H, sg); u += sg.yb - sg.ya + 1) {
                for (int r = sg.ya - 1; r <= sg.yb + 1; ++r, ++e) {
                    const uint32_t s = e % G::XR, t = e % G::TR;
                    if (!wait_or_abort(&xready[s], (e / G::XR) & 1u, &s_abort, p.err, 0xa3) ||
                        !wait_or_abort(&aempty[t], ((e / G::TR) & 1u) ^ 1u, &s_abort, p.err, 0xa4)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ar = desc_add(da, s * G::ROWB);
#pragma unroll
                    for (int ks = 0; ks < C / 16; ++ks)
                        mma_f16(tmem + t * U, desc_add(ar, ks * 2 * G::KGB), desc_add(db, ks * 256), idesc,
                                ks > 0 ? 1u : 0u);
                    mma_commit(&afull[t]);
                    mma_commit(&xfree[s]);
                }
            }
            mma_commit(&bar_end);  // every MMA has completed before TMEM is released
            mbar_wait(&bar_end, 0, 5000000ull);
        }
    } else if (warp < kDw0) {
        // ------------------------------ conv1 epilogue -----------------------
        const int q = warp & 3;  // TMEM lane quarter
        const int px = q * 32 + lane;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
        uint32_t e = 0;
        bool ok = true;
        for (long long u = u0; ok && seg_at(u, u1, H, sg); u += sg.yb - sg.ya + 1) {
            const int xg = sg.strip * G::OW - 1 + px;
            for (int r = sg.ya - 1; r <= sg.yb + 1; ++r, ++e) {
                const uint32_t t = e % G::TR, us = e % G::UR;
                const bool valid = r >= 0 && r < H && xg >= 0 && xg < W;
                ok = __all_sync(0xffffffffu, wait_or_abort(&afull[t], (e / G::TR) & 1u, &s_abort, p.err, 0xa5) &&
                                                 wait_or_abort(&ufree[us], ((e / G::UR) & 1u) ^ 1u, &s_abort,
                                                               p.err, 0xa6));
                if (!ok) break;
                tc_fence_after();
                uint8_t* dst = sU + us * G::UROWB + px * G::UPX;
#pragma unroll
                for (int c0 = 0; c0 < U; c0 += 32) {
                    float v[32];
                    tmem_ld16(lane_base + t * U + c0, *reinterpret_cast<float(*)[16]>(v));
                    tmem_ld16(lane_base + t * U + c0 + 16, *reinterpret_cast<float(*)[16]>(v + 16));
                    tmem_ld_wait();
                    if (c0 + 32 >= U) {  // the accumulator is drained
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&aempty[t]);
                    }
#pragma unroll
                    for (int j = 0; j < 32; j += 8) {
                        float f[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) f[i] = valid ? v[j + i] + sB1[c0 + j + i] : 0.f;
                        *reinterpret_cast<uint4*>(dst + (c0 + j) * 2) = f_to_h8(f);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&ufull[us]);
            }
        }
    } else {
        // ------------------------------ depthwise + gate ---------------------
        const int dwarp = warp - kDw0;
        const int pair = lane % G::PAIRS, grp = lane / G::PAIRS;
        const int walker = dwarp * G::GROUPS + grp;
        const int j0 = walker * G::OW / G::WALKERS, j1 = (walker + 1) * G::OW / G::WALKERS;
        const int ca = 2 * pair, cb = D + 2 * pair;  // u channels of the gate halves
        float2 ta[9], tb[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) {
            ta[k] = make_float2(sTap[k * U + ca], sTap[k * U + ca + 1]);
            tb[k] = make_float2(sTap[k * U + cb], sTap[k * U + cb + 1]);
        }
        const float2 ba = make_float2(sDwB[ca], sDwB[ca + 1]), bb = make_float2(sDwB[cb], sDwB[cb + 1]);
        float2 pool = make_float2(0.f, 0.f);
        uint32_t eb = 0, waited = 0;  // entry of the segment's first input row; entries < waited are ready
        bool ok = true;
        for (long long u = u0; ok && seg_at(u, u1, H, sg); u += sg.yb - sg.ya + 1) {
            const int x0 = sg.strip * G::OW;
            for (int y = sg.ya; y <= sg.yb; ++y) {
                const uint32_t e0 = eb + static_cast<uint32_t>(y - sg.ya);  // input row y - 1
                bool got = true;
                for (uint32_t e = max(waited, e0); e < e0 + 3; ++e)
                    got = got && wait_or_abort(&ufull[e % G::UR], (e / G::UR) & 1u, &s_abort, p.err, 0xa7);
                ok = __all_sync(0xffffffffu, got);
                if (!ok) break;
                waited = e0 + 3;
                const uint8_t* rows[3] = {sU + (e0 % G::UR) * G::UROWB, sU + ((e0 + 1) % G::UR) * G::UROWB,
                                          sU + ((e0 + 2) % G::UR) * G::UROWB};
                // window[row][col]: u of pixels j .. j+2 (columns x0+j-1 .. x0+j+1)
                float2 wa[3][3], wb[3][3];
                auto load_col = [&](int upx, int col) {
#pragma unroll
                    for (int k = 0; k < 3; ++k) {
                        const uint8_t* b = rows[k] + upx * G::UPX;
                        wa[k][col] = unpack_half2(*reinterpret_cast<const uint32_t*>(b + ca * 2));
                        wb[k][col] = unpack_half2(*reinterpret_cast<const uint32_t*>(b + cb * 2));
                    }
                };
                if (j0 < j1) {
                    load_col(j0, 0);
                    load_col(j0 + 1, 1);
                }
                __half* grow = p.g + (static_cast<size_t>(y) * W + x0) * D + ca;
                for (int j = j0; j < j1; ++j) {
                    load_col(j + 2, 2);
                    float2 aa = ba, ab = bb;
#pragma unroll
                    for (int k = 0; k < 3; ++k)
#pragma unroll
                        for (int c = 0; c < 3; ++c) {
                            aa = ffma2(wa[k][c], ta[k * 3 + c], aa);
                            ab = ffma2(wb[k][c], tb[k * 3 + c], ab);
                        }
                    const uint32_t h = pack_half2(aa.x * ab.x, aa.y * ab.y);
                    if (x0 + j < W) {
                        *reinterpret_cast<uint32_t*>(grow + static_cast<size_t>(j) * D) = h;
                        const float2 hf = unpack_half2(h);  // pool the stored fp16 values
                        pool.x += hf.x;
                        pool.y += hf.y;
                    }
#pragma unroll
                    for (int k = 0; k < 3; ++k) {
                        wa[k][0] = wa[k][1];
                        wa[k][1] = wa[k][2];
                        wb[k][0] = wb[k][1];
                        wb[k][1] = wb[k][2];
                    }
                }
                // u row y - 1 is used for the last time; at the segment's end
                // rows y and y + 1 too.
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&ufree[e0 % G::UR]);
                    if (y == sg.yb) {
                        mbar_arrive(&ufree[(e0 + 1) % G::UR]);
                        mbar_arrive(&ufree[(e0 + 2) % G::UR]);
                    }
                }
            }
            eb += static_cast<uint32_t>(sg.yb - sg.ya + 3);
        }
        // Pool: the walkers of a pair add in group order, then the warps in
        // warp order (fixed, deterministic).
        float px_ = pool.x, py_ = pool.y;
#pragma unroll
        for (int g = 1; g < G::GROUPS; ++g) {
            px_ += __shfl_down_sync(0xffffffffu, pool.x, g * G::PAIRS);
            py_ += __shfl_down_sync(0xffffffffu, pool.y, g * G::PAIRS);
        }
        if (grp == 0) {
            sPool[dwarp * D + ca] = px_;
            sPool[dwarp * D + ca + 1] = py_;
        }
    }

    __syncthreads();
    for (int c = tid; c < D; c += kSpThreads) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kDwWarps; ++w) s += sPool[w * D + c];
        p.partials[static_cast<size_t>(blockIdx.x) * D + c] = s;
    }
    if (p.b3_dst) sca_fold_last_cta<C, D, kSpThreads>(p, reinterpret_cast<float*>(sU), tid, warp, lane);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, G::TMEM_COLS);
}

template <int C>
int run_split(const FusedAParams& p, int grid, cudaStream_t s) {
    using G = SplitGeo<C>;
    static bool cfg = false;
    if (!cfg) {
        cudaError_t e = cudaFuncSetAttribute(split_a_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM);
        if (e != cudaSuccess) return dn_cuda_fail(e, "split phase A: smem attribute");
        cfg = true;
    }
    cudaError_t e = launch_pdl(split_a_kernel<C>, dim3(grid), dim3(kSpThreads), G::SMEM, s, p);
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "split phase A: launch");
}

}  // namespace

bool fused_a_split_supported(int C, int D, int N) { return (C == 32 || C == 64) && D == C && N == 1; }

int fused_a_split_grid(int C, int H, int W) {
    const long long units = static_cast<long long>((W + 125) / 126) * H;
    (void)C;
    return static_cast<int>(std::max(1LL, std::min<long long>(units, sm_count())));
}

int launch_fused_a_split(const FusedAParams& p, int C, int D, int grid, cudaStream_t s) {
    if (!fused_a_split_supported(C, D, p.N)) return dn_fail(DN_ERR_UNSUPPORTED, "split phase A: configuration");
    if (!p.w1 || !p.c2 || !p.dw_w || !p.dw_b) return dn_fail(DN_ERR_INVALID_ARG, "split phase A: missing weights");
    if (p.b3_dst && (!p.counter || !p.sca_w || !p.sca_b || !p.b3_src))
        return dn_fail(DN_ERR_INVALID_ARG, "split phase A: the SCA fold needs a counter and the SCA weights");
    if ((reinterpret_cast<uintptr_t>(p.x) & 15) || (reinterpret_cast<uintptr_t>(p.g) & 15))
        return dn_fail(DN_ERR_INVALID_ARG, "split phase A: x and g must be 16-byte aligned");
    if (C == 32) return run_split<32>(p, grid, s);
    return run_split<64>(p, grid, s);
}

}  // namespace dnb
