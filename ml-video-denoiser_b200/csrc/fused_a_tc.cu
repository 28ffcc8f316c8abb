// Strip-walking 3x3 convolutions on the tensor cores (C = 32 / 64 input
// channels): phase A of a shallow NAFBlock (below) and, with the same
// producer, row ring and MMA issuer, the model's ending conv (C -> 3 outputs
// padded to N = 16, plain zero padding and bias, the rows' LayerNorm replaced
// by a plain relayout; the epilogue crops, adds the beauty channels and
// writes NCHW; replaces the reference's ending cudnnConvolutionForward and
// the residual add, src/models/nafnet.cu:375-388).
//
// Phase A:
// LayerNorm1 (normalisation only), conv1 (1x1, C -> 2D) and the depthwise
// 3x3 conv (2D channels) compose into one linear map of the normalised input,
// so they run as a single 3x3 implicit GEMM over the normalised rows:
//   dw(u)[p, o] = bias_p[o] + sum_t sum_c Weff[t][o][c] * n[p + t, c],
//   Weff[t][o][c] = dw[o][t] * W1[o][c] * gamma1[c],
//   bias_p[o]    = b_dw[o] + b1'[o] * sum_{t: p + t inside the image} dw[o][t],
//   b1'[o]       = b1[o] + sum_c beta1[c] * W1[o][c],
// where n = (x - mean) * rstd is zero outside the image. The reference's
// depthwise zero padding of u therefore only masks bias taps: the kernel
// keeps the bias of each of the 16 tap-mask classes (interior, edges,
// corners) and every pixel looks its class up.
//
// A CTA owns a contiguous run of output rows of 128-pixel strips:
//   warp 0      producer: one input row (the strip's 128 pixels and the
//               1-pixel halo, contiguous in NHWC) per ring slot by one bulk
//               copy; rows outside the image are zeroed instead of loaded
//               (a tensor map with 16-byte inner boxes, which would write the
//               MMA layout directly, moves a row many times slower);
//   warps 1-4   LayerNorm of each row (FP32 statistics, FP16 result, as the
//               reference's normalised tensor) into the no-swizzle K-major
//               layout [C/8][130][8]. At 64 channels the four warps share a
//               row and write it back in place; at 32 channels the producer
//               lands rows in a second (pixel-major) ring and each warp
//               normalises whole rows on its own (a lane per pixel, no
//               shuffles), so four rows are in flight at once;
//   warp 5      MMA issuer, into a ring of TMEM accumulators (M = 128, the
//               strip's pixels; K = 16). At 32 channels, per input row r, 3
//               tap columns x C/16 K steps of N = 3 x 2D: the row's
//               contributions to output rows r-1, r, r+1 (taps ky = 2, 1, 0)
//               in one MMA. At 64 channels (N = 128 MMAs already run at the
//               tensor core's rate), per output row, 9 taps x C/16 K steps of
//               N = 2D. Tap column kx reads an input row from pixel kx on (a
//               16-byte shift of the start address), so each input row is
//               normalised once;
//   warps 6-9   epilogue: bias, SimpleGate, g stored straight from
//               registers (64 or 128 contiguous bytes per pixel), per-pixel
//               pool sums reduced in a fixed order (deterministic).
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
#include "sca_fold.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "sm100.cuh"
#include "status.h"

namespace dnb {
namespace {

constexpr int kTcThreads = 320;
constexpr int kMaxImg = 8;

// MODE 0: phase A of a NAFBlock (LN + conv1 + depthwise, SimpleGate, pool);
// MODE 1: the model's ending conv (C -> 3 outputs, padded to N = 16), cropped
// and added to the beauty channels.
template <int C, int MODE = 0>
struct GeoT {
    static constexpr int D = C;                         // gated channels (phase A)
    static constexpr int N = MODE == 0 ? 2 * C : 16;    // conv outputs per pixel
    static constexpr int SW = 128;             // strip width = MMA M
    static constexpr int HP = SW + 2;          // input pixels per row (halo)
    static constexpr int KG = C / 8;           // 16-byte channel groups
    static constexpr int KGB = HP * 16;        // bytes per channel group of a row (LBO)
    static constexpr int ROWB = KG * KGB;      // one input-row slot
    // At 32 channels (phase A and the ending) two CTAs run per SM (two
    // row pipelines, so that one's latencies overlap the other's), each with
    // half of TMEM and a 4-slot row ring.
    static constexpr int CTAS = C == 32 ? 2 : 1;
    static constexpr int R = (C >= 64 || CTAS == 2) ? 4 : 8;  // input-row slots (a power of two)
    static constexpr int KS = C / 16;          // K = 16 steps per tap
    static constexpr int TAPB = N * 32;        // B tile of one (tap, K step): 2D rows x 16
    static constexpr int WB = 9 * KS * TAPB;   // all of Weff
    static constexpr int ACC = 512 / N / CTAS;  // TMEM accumulator ring (all of the CTA's share)
    static constexpr int TMEM_COLS = ACC * N;
    // floats: bias per tap-mask class [16][N], pool sums [img][warp][D] (phase A)
    static constexpr int F_FLOATS = 16 * N + (MODE == 0 ? kMaxImg * 4 * D : 0);
    // At 32 channels each LayerNorm warp owns whole rows (WR): the producer
    // lands rows in a separate pixel-major ring, the warp writes the MMA
    // layout into the row ring, so four rows are normalised at once.
    static constexpr bool WR = C == 32;
    static constexpr int RAWB = WR ? R * ROWB : 0;
    // At least half of the SM's shared memory: the CTA holds all of TMEM, so a
    // second CTA on the same SM could only wait for it.
    static constexpr int SMEM_USED = 1024 + R * ROWB + WB + F_FLOATS * 4 + RAWB;
    static constexpr int SMEM = (CTAS == 2 || SMEM_USED > 120 * 1024) ? SMEM_USED : 120 * 1024;
    static_assert(ROWB % 128 == 0, "row slots stay 128-byte aligned");
    static_assert(TMEM_COLS <= 512, "TMEM ring");
    static_assert((R & (R - 1)) == 0 && (ACC & (ACC - 1)) == 0, "ring sizes are powers of two");
};

struct Seg {
    int img, strip, ya, yb;
};

// The segment starting at unit u of [u, u1): units enumerate (image, strip,
// output row) with rows fastest; a segment is the run of rows of one strip.
// Units are 32-bit: the launchers reject inputs with 2^31 units or more.
__device__ __forceinline__ bool seg_at(int u, int u1, int H, int strips, Seg& s) {
    if (u >= u1) return false;
    const int per_img = strips * H;
    s.img = u / per_img;
    const int rem = u - s.img * per_img;
    s.strip = rem / H;
    s.ya = rem - s.strip * H;
    s.yb = min(H - 1, s.ya + (u1 - u) - 1);
    return true;
}

// MMAs of one input row whose three output rows all belong to the strip
// segment (every row but the segment's first and last), with everything but
// the base addresses known at compile time: the issuing thread is on the
// kernel's critical path, and runtime operand arithmetic per MMA costs several
// times an N=64 MMA. tq[q] = TMEM address of output row r-1+q; PAT gives the
// MMA ranges of positions, split where the slots wrap around the ring:
// 0 = [0,3), 1 = [0,2)[2,3), 2 = [0,1)[1,3). The row's first (kx, K step)
// writes position 2 (the first contribution to output row r+1) with
// accumulate off.
template <int C, int MODE, int PAT>
__device__ __forceinline__ void issue_steady_row(const uint32_t (&tq)[3], uint64_t ar, uint64_t db) {
    using G = GeoT<C, MODE>;
    constexpr int N = G::N;
    static_assert(PAT != 0 || 3 * N <= 256, "three positions fit one MMA only at N <= 85");
#pragma unroll
    for (int kx = 0; kx < 3; ++kx)
#pragma unroll
        for (int ks = 0; ks < G::KS; ++ks) {
            const bool first = kx == 0 && ks == 0;
            const uint64_t a = desc_add(ar, ks * 2 * G::KGB + kx * 16);
            const uint64_t b = desc_add(db, (kx * G::KS + ks) * 3 * G::TAPB);
            if (PAT == 0) {
                if (first) {
                    mma_f16(tq[0], a, b, idesc_f16_f32(128, 2 * N), 1u);
                    mma_f16(tq[2], a, desc_add(b, 2 * G::TAPB), idesc_f16_f32(128, N), 0u);
                } else {
                    mma_f16(tq[0], a, b, idesc_f16_f32(128, 3 * N), 1u);
                }
            } else if (PAT == 1) {
                mma_f16(tq[0], a, b, idesc_f16_f32(128, 2 * N), 1u);
                mma_f16(tq[2], a, desc_add(b, 2 * G::TAPB), idesc_f16_f32(128, N), first ? 0u : 1u);
            } else {
                mma_f16(tq[0], a, b, idesc_f16_f32(128, N), 1u);
                if (first) {
                    mma_f16(tq[1], a, desc_add(b, G::TAPB), idesc_f16_f32(128, N), 1u);
                    mma_f16(tq[2], a, desc_add(b, 2 * G::TAPB), idesc_f16_f32(128, N), 0u);
                } else {
                    mma_f16(tq[1], a, desc_add(b, G::TAPB), idesc_f16_f32(128, 2 * N), 1u);
                }
            }
        }
}

__device__ __forceinline__ float finite_or_zero(float v) { return (isnan(v) || isinf(v)) ? 0.f : v; }

// P = FusedAParams (MODE 0) or EndingParams (MODE 1): the conv input is
// in_h x in_w (NHWC, C channels), the outputs cover out_h x out_w.
template <int C, int MODE, class P>
__global__ void __launch_bounds__(kTcThreads, GeoT<C, MODE>::CTAS) tc_conv_kernel(const __grid_constant__ P p) {
    using G = GeoT<C, MODE>;
    constexpr int D = G::D, N = G::N;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sRow = smem;                                 // R input-row slots
    uint8_t* sW = sRow + G::R * G::ROWB;                  // Weff B tiles
    // Bias of a pixel by the taps whose input lies outside the image: class
    // bits 0/1 = left/right column invalid, bits 2/3 = top/bottom row invalid
    // (class 0 = interior).
    float* sBias = reinterpret_cast<float*>(sW + G::WB);  // [16][N]
    float* sPool = sBias + 16 * N;                        // [img][epilogue warp][D]
    uint8_t* sRaw = reinterpret_cast<uint8_t*>(sPool + (MODE == 0 ? kMaxImg * 4 * D : 0));  // WR: R pixel-major rows
    __shared__ uint64_t full[G::R], ready[G::R], freeb[G::R], rawfree[G::R], acc_full[G::ACC], acc_empty[G::ACC];
    __shared__ uint64_t bar_w, bar_end;
    __shared__ uint32_t tslot;
    __shared__ volatile int s_abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int in_h, in_w, out_h, out_w;
    if constexpr (MODE == 0) {
        in_h = out_h = p.H;
        in_w = out_w = p.W;
    } else {
        in_h = p.Hp;
        in_w = p.Wp;
        out_h = p.H;
        out_w = p.W;
    }
    const int strips = (out_w + G::SW - 1) / G::SW;
    const long long T = static_cast<long long>(p.N) * strips * out_h;
    const int u0 = static_cast<int>(T * blockIdx.x / gridDim.x), u1 = static_cast<int>(T * (blockIdx.x + 1) / gridDim.x);

    for (int i = tid; i < 16 * N; i += kTcThreads) {
        const int cls = i / N, o = i - cls * N;
        if constexpr (MODE == 0) {
            float sum = 0.f;
#pragma unroll
            for (int tp = 0; tp < 9; ++tp) {
                const int ky = tp / 3, kx = tp % 3;
                const bool off = (kx == 0 && (cls & 1)) || (kx == 2 && (cls & 2)) || (ky == 0 && (cls & 4)) ||
                                 (ky == 2 && (cls & 8));
                if (!off) sum += p.dw_w[tp * N + o];
            }
            sBias[i] = fmaf(p.b1p[o], sum, p.dw_b[o]);
        } else {
            sBias[i] = o < 3 ? p.b[o] : 0.f;  // a plain conv bias: no tap mask
        }
    }
    if constexpr (MODE == 0)
        for (int i = tid; i < kMaxImg * 4 * D; i += kTcThreads) sPool[i] = 0.f;
    if (warp == 0) {
        tmem_alloc(&tslot, G::TMEM_COLS);
        tmem_relinquish();
    }
    if (tid == 0) {
        for (int s = 0; s < G::R; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&ready[s], G::WR ? 1 : 4);
            mbar_init(&freeb[s], 1);
            mbar_init(&rawfree[s], 1);
        }
        for (int a = 0; a < G::ACC; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], 4);
        }
        mbar_init(&bar_w, 1);
        mbar_init(&bar_end, 1);
        s_abort = 0;
        fence_mbar_init();
        mbar_arrive_expect_tx(&bar_w, G::WB);
        bulk_g2s(sW, p.weff, G::WB, &bar_w);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    pdl_trigger();  // only once this CTA holds its TMEM columns
    pdl_wait();  // x was written by the previous kernel; g and the partials are read by it

    Seg sg;
    if (warp == 0) {
        // ------------------------------ producer -----------------------------
        if (lane == 0) {
            uint32_t e = 0;
            for (int u = u0; !s_abort && seg_at(u, u1, out_h, strips, sg); u += sg.yb - sg.ya + 1) {
                const int x0 = sg.strip * G::SW;
                for (int r = sg.ya - 1; r <= sg.yb + 1; ++r, ++e) {
                    const uint32_t s = e % G::R, ph = (e / G::R) & 1u;
                    // WR: the raw slot is free once its LayerNorm warp has read it;
                    // otherwise the row slot is reused in place, free once its MMAs
                    // have completed.
                    if (!wait_or_abort(G::WR ? &rawfree[s] : &freeb[s], ph ^ 1u, &s_abort, p.err, 0x70)) break;
                    if (r < 0 || r >= in_h) {
                        mbar_arrive(&full[s]);  // zeroed by the LayerNorm warps
                    } else {
                        // The strip's input pixels [x0-1, x0+129) clipped to the
                        // image are contiguous in NHWC: one bulk copy, landing
                        // pixel-major at their slot positions.
                        const int pa = max(0, x0 - 1), pb = min(in_w, x0 + G::SW + 1);
                        const uint32_t bytes = static_cast<uint32_t>(pb - pa) * C * 2;
                        mbar_arrive_expect_tx(&full[s], bytes);
                        bulk_g2s((G::WR ? sRaw : sRow) + s * G::ROWB + (pa - (x0 - 1)) * C * 2,
                                 p.x + ((static_cast<size_t>(sg.img) * in_h + r) * in_w + pa) * C, bytes, &full[s]);
                    }
                }
            }
            if (s_abort) {
                // Let the copies already issued land before the CTA's memory is released.
                for (uint32_t k = e > G::R ? e - G::R : 0; k < e; ++k)
                    mbar_wait(&full[k % G::R], (k / G::R) & 1u, 5000000ull);
            }
        }
    } else if (warp <= 4) {
      if constexpr (G::WR) {
        // ------------------------- LayerNorm, a row per warp -----------------
        // Warp w takes the ring entries e = w (mod 4) (slot e mod R). A lane
        // owns pixels lane + 32k of the row: its statistics need no shuffles.
        // It reads the pixel's four 16-byte chunks in a lane-rotated order
        // (conflict-free pixel-major reads) and writes each normalised chunk
        // to its place in the MMA layout [C/8][130][8 ch] of the row slot,
        // once the MMAs of that slot's previous row have completed.
        static_assert(G::R == 4 && C == 32, "one slot per LayerNorm warp");
        const int w = warp - 1;
        const int rot = (lane >> 1) & 3;
        uint32_t e = 0;
        bool ok = true;
        for (int u = u0; ok && seg_at(u, u1, out_h, strips, sg); u += sg.yb - sg.ya + 1) {
            const int x0 = sg.strip * G::SW;
            for (int r = sg.ya - 1; r <= sg.yb + 1; ++r, ++e) {
                if (static_cast<int>(e & 3u) != w) continue;
                const uint32_t s = e % G::R, ph = (e / G::R) & 1u;
                ok = __all_sync(0xffffffffu, wait_or_abort(&full[s], ph, &s_abort, p.err, 0x71));
                if (ok) ok = __all_sync(0xffffffffu, wait_or_abort(&freeb[s], ph ^ 1u, &s_abort, p.err, 0x76));
                if (!ok) break;
                const uint8_t* raw = sRaw + s * G::ROWB;
                uint8_t* row = sRow + s * G::ROWB;
                const bool row_in = r >= 0 && r < in_h;
                constexpr int NP = (G::HP + 31) / 32;  // pixel passes
#pragma unroll 1
                for (int k = 0; k < NP; ++k) {
                    const int i = k * 32 + lane;
                    const int xin = x0 - 1 + i;
                    const bool valid = row_in && i < G::HP && xin >= 0 && xin < in_w;
                    uint4 cur[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        cur[q] = valid ? *reinterpret_cast<const uint4*>(raw + i * 64 + ((q + rot) & 3) * 16)
                                       : make_uint4(0u, 0u, 0u, 0u);
                    if constexpr (MODE == 0) {
                        // Sums and sums of squares of the pixel's 32 channels (fp32;
                        // zero rows and pixels outside the image stay zero).
                        const float2 one = make_float2(1.f, 1.f);
                        float2 a1 = make_float2(0.f, 0.f), a2 = make_float2(0.f, 0.f);
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const uint32_t wv[4] = {cur[q].x, cur[q].y, cur[q].z, cur[q].w};
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const float2 d = unpack_half2(wv[j]);
                                a1 = ffma2(d, one, a1);
                                a2 = ffma2(d, d, a2);
                            }
                        }
                        const float dm = (a1.x + a1.y) * (1.0f / C);
                        const float var = fmaxf((a2.x + a2.y) * (1.0f / C) - dm * dm, 0.f);
                        const float rstd = rsqrtf(var + 1e-6f);
                        const float2 rs2 = make_float2(rstd, rstd);
                        const float2 sh2 = make_float2(-dm * rstd, -dm * rstd);
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const uint32_t wv[4] = {cur[q].x, cur[q].y, cur[q].z, cur[q].w};
                            uint32_t o[4];
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const float2 y = ffma2(unpack_half2(wv[j]), rs2, sh2);
                                o[j] = pack_half2(y.x, y.y);
                            }
                            cur[q] = valid ? make_uint4(o[0], o[1], o[2], o[3]) : make_uint4(0u, 0u, 0u, 0u);
                        }
                    }
                    if (i < G::HP) {
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            *reinterpret_cast<uint4*>(row + ((q + rot) & 3) * G::KGB + i * 16) = cur[q];
                    }
                }
                fence_async_smem();  // the tensor core reads the row (async proxy)
                __syncwarp();        // every lane has read the raw row and written its chunks
                if (lane == 0) {
                    mbar_arrive(&rawfree[s]);
                    mbar_arrive(&ready[s]);
                }
            }
        }
      } else {
        // ------------------------------ LayerNorm ----------------------------
        // A pixel's C/8 16-byte chunks sit in adjacent lanes (conflict-free
        // reads of the pixel-major row); its statistics (sum and sum of
        // squares) are reduced over those lanes. The normalised
        // row stays in registers until all 128 threads have read the slot, then
        // is written back in the MMA layout [C/8][130][8 ch].
        constexpr int CPX = C / 8, PPR = 128 / CPX, NR = (G::HP + PPR - 1) / PPR;
        const int t = tid - 32;
        const int cq = t % CPX, pl = t / CPX;
        uint32_t e = 0;
        bool ok = true;
        for (int u = u0; ok && seg_at(u, u1, out_h, strips, sg); u += sg.yb - sg.ya + 1) {
            const int x0 = sg.strip * G::SW;
            for (int r = sg.ya - 1; r <= sg.yb + 1; ++r, ++e) {
                const uint32_t s = e % G::R, ph = (e / G::R) & 1u;
                // One decision for all four LayerNorm warps: they meet at the
                // named barrier below, so none may leave the loop alone.
                const bool got = wait_or_abort(&full[s], ph, &s_abort, p.err, 0x71);
                if (named_sync_or(1, 128, !got)) {
                    ok = false;
                    break;
                }
                uint8_t* row = sRow + s * G::ROWB;
                const bool row_in = r >= 0 && r < in_h;
                // Phases over the NR pixel passes, so that their latency chains
                // overlap: every load, then the partial sums, the lane
                // reductions interleaved across passes, the rsqrts, and the
                // normalisation.
                uint4 nv[NR];
                bool valid[NR];
#pragma unroll
                for (int k = 0; k < NR; ++k) {
                    const int i = k * PPR + pl;
                    const int xin = x0 - 1 + i;
                    valid[k] = row_in && i < G::HP && xin >= 0 && xin < in_w;
                    nv[k] = valid[k] ? *reinterpret_cast<const uint4*>(row + i * C * 2 + cq * 16)
                                     : make_uint4(0u, 0u, 0u, 0u);
                }
                if constexpr (MODE == 0) {
                    // Sums and sums of squares of the pixel's channels (fp32 over C
                    // values: E[x^2] - mean^2 loses nothing at these sizes).
                    float s1[NR], s2[NR];
                    const float2 one = make_float2(1.f, 1.f);
#pragma unroll
                    for (int k = 0; k < NR; ++k) {
                        const uint32_t w[4] = {nv[k].x, nv[k].y, nv[k].z, nv[k].w};
                        float2 a1 = make_float2(0.f, 0.f), a2 = make_float2(0.f, 0.f);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float2 d = unpack_half2(w[j]);
                            a1 = ffma2(d, one, a1);
                            a2 = ffma2(d, d, a2);
                        }
                        s1[k] = a1.x + a1.y;
                        s2[k] = a2.x + a2.y;
                    }
#pragma unroll
                    for (int m = 1; m < CPX; m <<= 1) {
#pragma unroll
                        for (int k = 0; k < NR; ++k) {
                            s1[k] += __shfl_xor_sync(0xffffffffu, s1[k], m);
                            s2[k] += __shfl_xor_sync(0xffffffffu, s2[k], m);
                        }
                    }
#pragma unroll
                    for (int k = 0; k < NR; ++k) {
                        const float dm = s1[k] * (1.0f / C);
                        const float var = fmaxf(s2[k] * (1.0f / C) - dm * dm, 0.f);
                        const float rstd = rsqrtf(var + 1e-6f);
                        const float2 rs2 = make_float2(rstd, rstd);
                        const float2 sh2 = make_float2(-dm * rstd, -dm * rstd);
                        const uint32_t w[4] = {nv[k].x, nv[k].y, nv[k].z, nv[k].w};
                        uint32_t o[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float2 y = ffma2(unpack_half2(w[j]), rs2, sh2);
                            o[j] = pack_half2(y.x, y.y);
                        }
                        nv[k] = valid[k] ? make_uint4(o[0], o[1], o[2], o[3]) : make_uint4(0u, 0u, 0u, 0u);
                    }
                }
                named_sync(1, 128);  // every thread has read the pixel-major row
#pragma unroll
                for (int k = 0; k < NR; ++k) {
                    const int i = k * PPR + pl;
                    if (i < G::HP) *reinterpret_cast<uint4*>(row + cq * G::KGB + i * 16) = nv[k];
                }
                fence_async_smem();  // the tensor core reads the row (async proxy)
                __syncwarp();
                if (lane == 0) mbar_arrive(&ready[s]);
            }
        }
      }
    } else if (warp == 5) {
      if constexpr (3 * N <= 256) {
        // ------------------------------ MMA issuer ---------------------------
        // Input row r feeds output rows r-1, r, r+1 (taps ky = 2, 1, 0). The B
        // tile of (kx, K step) stacks [W(ky=2) | W(ky=1) | W(ky=0)] along N, so
        // one MMA over positions q = 0..2 adds the row into the three output
        // rows' accumulators, which sit in consecutive TMEM slots (the output
        // row of running index j in slot j mod ACC). An MMA is split where the
        // slots wrap around the ring, where N would pass 256, and, for the
        // row's first (kx, K step), before position 2: that is the first
        // contribution to output row r+1 (accumulate off), so no slot needs
        // zeroing. Output row r-1 is complete once row r has been issued.
        if (lane == 0) {
            constexpr int MAXQ = 256 / N < 3 ? 256 / N : 3;  // positions per MMA
            const uint64_t da = sdesc_kmajor(smem_u32(sRow), G::KGB, 128);
            const uint64_t db = sdesc_kmajor(smem_u32(sW), 128, 256);
            bool ok = wait_or_abort(&bar_w, 0, &s_abort, p.err, 0x72);
            uint32_t e = 0, rb = 0;  // entry counter; running index of the segment's first output row
            for (int u = u0; ok && seg_at(u, u1, out_h, strips, sg); u += sg.yb - sg.ya + 1) {
                for (int r = sg.ya - 1; r <= sg.yb + 1; ++r, ++e) {
                    const uint32_t s_in = e & (G::R - 1);
                    if (!wait_or_abort(&ready[s_in], (e / G::R) & 1u, &s_abort, p.err, 0x73)) {
                        ok = false;
                        break;
                    }
                    // Positions whose output row r - 1 + q lies in [ya, yb].
                    const int qlo = max(0, sg.ya - (r - 1)), qhi = min(3, sg.yb - (r - 1) + 1);
                    const int j0 = static_cast<int>(rb) + (r - 1 - sg.ya);  // running index at q = 0
                    if (qhi == 3) {  // output row r + 1 starts: its slot must be drained
                        const uint32_t j2 = static_cast<uint32_t>(j0 + 2);
                        if (!wait_or_abort(&acc_empty[j2 & (G::ACC - 1)], ((j2 / G::ACC) & 1u) ^ 1u, &s_abort, p.err,
                                           0x74)) {
                            ok = false;
                            break;
                        }
                    }
                    tc_fence_after();
                    const uint64_t ar = desc_add(da, s_in * G::ROWB);
                    if (qlo == 0 && qhi == 3) {
                        uint32_t tq[3];
#pragma unroll
                        for (int q = 0; q < 3; ++q) tq[q] = tmem + (static_cast<uint32_t>(j0 + q) & (G::ACC - 1)) * N;
                        const uint32_t p0 = static_cast<uint32_t>(j0) & (G::ACC - 1);
                        if (p0 == G::ACC - 1) {
                            issue_steady_row<C, MODE, 2>(tq, ar, db);
                        } else if (3 * N > 256 || p0 == G::ACC - 2) {
                            issue_steady_row<C, MODE, 1>(tq, ar, db);
                        } else {
                            issue_steady_row<C, MODE, (3 * N <= 256 ? 0 : 1)>(tq, ar, db);
                        }
                    } else {
                        // Segment edges: the general split, ranges [cut[i], cut[i+1]).
                        int cut[4], nc = 0;
                        cut[nc++] = qlo;
                        for (int q = qlo + 1; q < qhi; ++q)
                            if ((static_cast<uint32_t>(j0 + q) & (G::ACC - 1)) == 0 || q - cut[nc - 1] >= MAXQ)
                                cut[nc++] = q;
                        cut[nc] = qhi;
                        for (int kx = 0; kx < 3; ++kx)
                            for (int ks = 0; ks < G::KS; ++ks) {
                                const bool first = kx == 0 && ks == 0;
                                const uint64_t a = desc_add(ar, ks * 2 * G::KGB + kx * 16);
                                const uint64_t b0 = desc_add(db, (kx * G::KS + ks) * 3 * G::TAPB);
                                auto issue = [&](int qa, int qb, uint32_t acc_on) {
                                    const uint32_t slot = static_cast<uint32_t>(j0 + qa) & (G::ACC - 1);
                                    mma_f16(tmem + slot * N, a, desc_add(b0, qa * G::TAPB),
                                            idesc_f16_f32(128, (qb - qa) * N), acc_on);
                                };
                                for (int i = 0; i < nc; ++i) {
                                    const int qa = cut[i], qb = cut[i + 1];
                                    if (first && qa < 2 && qb > 2) {
                                        issue(qa, 2, 1u);
                                        issue(2, qb, 0u);
                                    } else {
                                        issue(qa, qb, (first && qa == 2) ? 0u : 1u);
                                    }
                                }
                            }
                    }
                    if (qlo == 0) mma_commit(&acc_full[static_cast<uint32_t>(j0) & (G::ACC - 1)]);
                    mma_commit(&freeb[s_in]);  // the row's only reader is done
                }
                rb += static_cast<uint32_t>(sg.yb - sg.ya + 1);
            }
            mma_commit(&bar_end);  // every MMA has completed before TMEM is released
            mbar_wait(&bar_end, 0, 5000000ull);
        }
      } else {
        // ------------------------------ MMA issuer ---------------------------
        // One output row at a time (64 channels: N = 128 MMAs already run at
        // the tensor core's rate, so the stacked form above gains nothing):
        // 9 taps x C/16 K steps into the row's accumulator; the B tile of tap
        // (ky, kx) sits at position 2 - ky of the stacked (kx, K step) tile.
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(128, N);
            const uint64_t da = sdesc_kmajor(smem_u32(sRow), G::KGB, 128);
            const uint64_t db = sdesc_kmajor(smem_u32(sW), 128, 256);
            bool ok = wait_or_abort(&bar_w, 0, &s_abort, p.err, 0x72);
            uint32_t eb = 0, rr = 0, waited = 0;  // entries < waited are known to be ready
            for (int u = u0; ok && seg_at(u, u1, out_h, strips, sg); u += sg.yb - sg.ya + 1) {
                for (int y = sg.ya; y <= sg.yb; ++y, ++rr) {
                    const uint32_t e0 = eb + static_cast<uint32_t>(y - sg.ya);
                    const uint32_t sl[3] = {e0 & (G::R - 1), (e0 + 1) & (G::R - 1), (e0 + 2) & (G::R - 1)};
                    // Rows y-1 and y were waited for by the previous output row
                    // of the segment: only new entries cost a barrier wait.
                    for (uint32_t e = max(waited, e0); ok && e < e0 + 3; ++e)
                        if (!wait_or_abort(&ready[e & (G::R - 1)], (e / G::R) & 1u, &s_abort, p.err, 0x73)) ok = false;
                    waited = e0 + 3;
                    const uint32_t a = rr & (G::ACC - 1);
                    if (ok && !wait_or_abort(&acc_empty[a], ((rr / G::ACC) & 1u) ^ 1u, &s_abort, p.err, 0x74))
                        ok = false;
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t acc = tmem + a * N;
#pragma unroll
                    for (int ky = 0; ky < 3; ++ky) {
                        const uint64_t ar = desc_add(da, sl[ky] * G::ROWB);
#pragma unroll
                        for (int kx = 0; kx < 3; ++kx)
#pragma unroll
                            for (int ks = 0; ks < G::KS; ++ks)
                                mma_f16(acc, desc_add(ar, ks * 2 * G::KGB + kx * 16),
                                        desc_add(db, ((kx * G::KS + ks) * 3 + (2 - ky)) * G::TAPB), idesc,
                                        (ky | kx | ks) ? 1u : 0u);
                    }
                    mma_commit(&acc_full[a]);
                    mma_commit(&freeb[sl[0]]);  // last use of input row y - 1
                    if (y == sg.yb) {           // the strip segment ends: rows y and y + 1 too
                        mma_commit(&freeb[sl[1]]);
                        mma_commit(&freeb[sl[2]]);
                    }
                }
                eb += static_cast<uint32_t>(sg.yb - sg.ya + 3);
            }
            mma_commit(&bar_end);  // every MMA has completed before TMEM is released
            mbar_wait(&bar_end, 0, 5000000ull);
        }
      }
    } else {
        // ------------------------------ epilogue -----------------------------
        const int q = warp & 3;  // TMEM lane quarter = pixels 32q .. 32q+31 of the strip
        const int px = q * 32 + lane;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
      if constexpr (MODE == 1) {
        // y = finite(beauty) + conv + bias for the first 3 outputs, inside the
        // crop, NCHW (a warp writes 32 consecutive pixels of each plane).
        uint32_t rr = 0;
        bool ok = true;
        const size_t plane = static_cast<size_t>(out_h) * out_w;
        for (int u = u0; ok && seg_at(u, u1, out_h, strips, sg); u += sg.yb - sg.ya + 1) {
            const int xg = sg.strip * G::SW + px;
            const bool col_ok = xg < out_w;
            const __half* bt = p.beauty + static_cast<size_t>(sg.img) * p.beauty_batch_stride;
            __half* yo = p.y + static_cast<size_t>(sg.img) * 3 * plane;
            // The beauty values of a row are loaded one row ahead: their
            // latency then overlaps the wait for the row's accumulator.
            auto beauty_row = [&](int y, __half (&bv)[3]) {
#pragma unroll
                for (int c = 0; c < 3; ++c)
                    bv[c] = col_ok ? bt[c * plane + static_cast<size_t>(y) * out_w + xg] : __float2half(0.f);
            };
            __half bcur[3];
            beauty_row(sg.ya, bcur);
            for (int y = sg.ya; y <= sg.yb; ++y, ++rr) {
                __half bnext[3];
                beauty_row(y < sg.yb ? y + 1 : y, bnext);
                const uint32_t a = rr & (G::ACC - 1);
                ok = __all_sync(0xffffffffu,
                                wait_or_abort(&acc_full[a], (rr / G::ACC) & 1u, &s_abort, p.err, 0x75));
                if (!ok) break;
                tc_fence_after();
                float v[16];
                tmem_ld16(lane_base + a * N, v);
                tmem_ld_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[a]);
                if (col_ok) {
                    const size_t o = static_cast<size_t>(y) * out_w + xg;
#pragma unroll
                    for (int c = 0; c < 3; ++c)
                        yo[c * plane + o] = __float2half(finite_or_zero(__half2float(bcur[c])) + (v[c] + sBias[c]));
                }
#pragma unroll
                for (int c = 0; c < 3; ++c) bcur[c] = bnext[c];
            }
        }
      } else {
        float ps[D];
#pragma unroll
        for (int c = 0; c < D; ++c) ps[c] = 0.f;
        // Pool sums of this warp's pixels -> sPool[img][q][:] (fixed order).
        auto flush = [&](int img) {
#pragma unroll
            for (int c = 0; c < D; ++c) {
                float v = ps[c];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
                if (lane == 0) sPool[(img * 4 + q) * D + c] += v;
                ps[c] = 0.f;
            }
        };
        uint32_t rr = 0;
        int cur = -1;
        bool ok = true;
        for (int u = u0; ok && seg_at(u, u1, out_h, strips, sg); u += sg.yb - sg.ya + 1) {
            if (cur >= 0 && sg.img != cur) flush(cur);
            cur = sg.img;
            const int xg = sg.strip * G::SW + px;
            const bool col_ok = xg < p.W;
            for (int y = sg.ya; y <= sg.yb; ++y, ++rr) {
                const uint32_t a = rr & (G::ACC - 1);
                ok = __all_sync(0xffffffffu,
                                wait_or_abort(&acc_full[a], (rr / G::ACC) & 1u, &s_abort, p.err, 0x75));
                if (!ok) break;
                tc_fence_after();
                // Tap mask of the bias: taps whose input pixel lies outside
                // the image contribute no conv1 bias (the DW zero padding).
                const int cls = (xg == 0 ? 1 : 0) | (xg == p.W - 1 ? 2 : 0) | (y == 0 ? 4 : 0) | (y == p.H - 1 ? 8 : 0);
                const float* bias_c = sBias + cls * N;
                __half* dst = p.g + ((static_cast<size_t>(sg.img) * p.H + y) * p.W + xg) * D;
                // EPW gate channels per pass: both halves' accumulator columns
                // (tcgen05.ld is warp-collective: every lane loads); 16 when
                // two CTAs share the SM's registers.
                constexpr int EPW = G::CTAS == 2 ? 16 : 32;
#pragma unroll
                for (int cc = 0; cc < D; cc += EPW) {
                    float va[EPW], vb[EPW];
#pragma unroll
                    for (int h = 0; h < EPW; h += 16) {
                        tmem_ld16(lane_base + a * N + cc + h, *reinterpret_cast<float(*)[16]>(va + h));
                        tmem_ld16(lane_base + a * N + D + cc + h, *reinterpret_cast<float(*)[16]>(vb + h));
                    }
                    tmem_ld_wait();
                    if (cc + EPW >= D) {  // the accumulator is drained
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&acc_empty[a]);
                    }
                    if (!col_ok) continue;
#pragma unroll
                    for (int c8 = 0; c8 < EPW; c8 += 8) {
                        const int c = cc + c8;
                        float bias[16];
#pragma unroll
                        for (int i = 0; i < 8; i += 4) {
                            const float4 ba = *reinterpret_cast<const float4*>(bias_c + c + i);
                            const float4 bb = *reinterpret_cast<const float4*>(bias_c + D + c + i);
                            bias[i] = ba.x;
                            bias[i + 1] = ba.y;
                            bias[i + 2] = ba.z;
                            bias[i + 3] = ba.w;
                            bias[8 + i] = bb.x;
                            bias[8 + i + 1] = bb.y;
                            bias[8 + i + 2] = bb.z;
                            bias[8 + i + 3] = bb.w;
                        }
                        float gv[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) gv[i] = (va[c8 + i] + bias[i]) * (vb[c8 + i] + bias[8 + i]);
                        const uint4 h = f_to_h8(gv);
                        *reinterpret_cast<uint4*>(dst + c) = h;
                        float hf[8];
                        h8_to_f(h, hf);  // pool the stored fp16 values
#pragma unroll
                        for (int i = 0; i < 8; ++i) ps[c + i] += hf[i];
                    }
                }
            }
        }
        if (cur >= 0) flush(cur);
      }
    }

    __syncthreads();
    if constexpr (MODE == 0) {
        for (int i = tid; i < p.N * D; i += kTcThreads) {
            const int n = i / D, c = i - n * D;
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < 4; ++w) s += sPool[(n * 4 + w) * D + c];
            p.partials[(static_cast<size_t>(n) * gridDim.x + blockIdx.x) * D + c] = s;
        }
        if (p.b3_dst) sca_fold_last_cta<C, D, kTcThreads>(p, sPool, tid, warp, lane);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, G::TMEM_COLS);
}

template <int C, int MODE, class P>
int run_tc(const P& p, int grid, cudaStream_t s) {
    using G = GeoT<C, MODE>;
    auto kern = tc_conv_kernel<C, MODE, P>;
    static bool cfg = false;
    if (!cfg) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM);
        if (e != cudaSuccess) return dn_cuda_fail(e, "tc conv: smem attribute");
        cfg = true;
    }
    cudaError_t e = launch_pdl(kern, dim3(grid), dim3(kTcThreads), G::SMEM, s, p);
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "tc conv: launch");
}

}  // namespace

bool fused_a_tc_supported(int C, int D) { return (C == 32 || C == 64) && D == C; }

int fused_a_tc_grid(int C, int N, int H, int W) {
    const long long units = static_cast<long long>(N) * ((W + 127) / 128) * H;
    const int per_sm = C == 32 ? GeoT<32, 0>::CTAS : GeoT<64, 0>::CTAS;
    return static_cast<int>(std::max(1LL, std::min<long long>(units, static_cast<long long>(sm_count()) * per_sm)));
}

int launch_fused_a_tc(const FusedAParams& p, int C, int D, int grid, cudaStream_t s) {
    if (p.N > kMaxImg) return dn_fail(DN_ERR_UNSUPPORTED, "fused_a_tc: batch > 8");
    if (!p.weff || !p.b1p) return dn_fail(DN_ERR_INVALID_ARG, "fused_a_tc: missing packed weights");
    if (p.b3_dst && (p.N != 1 || !p.counter || !p.sca_w || !p.sca_b || !p.b3_src))
        return dn_fail(DN_ERR_INVALID_ARG, "fused_a_tc: the SCA fold needs one image, a counter and the SCA weights");
    if ((reinterpret_cast<uintptr_t>(p.x) & 15) || (reinterpret_cast<uintptr_t>(p.g) & 15))
        return dn_fail(DN_ERR_INVALID_ARG, "fused_a_tc: x and g must be 16-byte aligned");
    if (static_cast<long long>(p.N) * ((p.W + 127) / 128) * p.H >= (1LL << 31))
        return dn_fail(DN_ERR_UNSUPPORTED, "fused_a_tc: too many strip rows");
    if (C == 32 && D == 32) return run_tc<32, 0>(p, grid, s);
    if (C == 64 && D == 64) return run_tc<64, 0>(p, grid, s);
    return dn_fail(DN_ERR_UNSUPPORTED, "fused_a_tc: channel configuration");
}

bool ending_tc_supported(int C0) { return C0 == 32 || C0 == 64; }

int launch_ending_tc(const EndingParams& p, cudaStream_t s) {
    if (!p.weff) return dn_fail(DN_ERR_INVALID_ARG, "ending_tc: missing packed weights");
    if ((reinterpret_cast<uintptr_t>(p.x) & 15)) return dn_fail(DN_ERR_INVALID_ARG, "ending_tc: x must be 16-byte aligned");
    const long long units = static_cast<long long>(p.N) * ((p.W + 127) / 128) * p.H;
    if (units >= (1LL << 31)) return dn_fail(DN_ERR_UNSUPPORTED, "ending_tc: too many strip rows");
    const int per_sm = p.C0 == 32 ? GeoT<32, 1>::CTAS : GeoT<64, 1>::CTAS;
    const int grid = static_cast<int>(std::max(1LL, std::min<long long>(units, static_cast<long long>(sm_count()) * per_sm)));
    if (p.C0 == 32) return run_tc<32, 1>(p, grid, s);
    if (p.C0 == 64) return run_tc<64, 1>(p, grid, s);
    return dn_fail(DN_ERR_UNSUPPORTED, "ending_tc: channel count");
}

}  // namespace dnb
