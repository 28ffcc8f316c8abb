// Persistent, warp-specialised implicit GEMM on the 5th-generation tensor
// cores (tcgen05):  out[M, N] = epi( pro(A)[M, K] * B[N, K]^T ).
//
// Roles (480 threads per CTA, one CTA owns a stream of 128 x NT tiles):
//   warp 12     A producer: per K-chunk, 2-D tensor-map loads of the A rows
//               (one 128-byte-swizzled box of KC channels, or 8-channel boxes
//               landing directly in the no-swizzle K-major UMMA layout: LBO
//               2 KB between 8-wide K groups, SBO 128 B between 8-row groups).
//   warp 14     B producer: one bulk copy of the pre-packed B tile per
//               K-chunk. Both arrive on the stage's `raw` mbarrier; two
//               issuing threads keep two copies in flight per stage.
//   warps 0-3   transform, thread t = tile row t:
//                 LayerNorm: accumulates the row statistics (shifted sums)
//                   from the staged chunks while the MMA consumes them - the
//                   LN itself is folded into the weights and the epilogue:
//                   LN(x) W^T = rstd * (x (gW)^T - mean * c1) + c2,
//                   c1[n] = sum_k (gW)[n,k], c2[n] = sum_k b_ln[k] W[n,k] + bias[n];
//                 SCA scale: A[m,k] *= s[img,k] in place before the MMA;
//                 2x2 stride-2 conv: gathers the patch rows itself.
//   warp 13     MMA issuer: one thread issues KC/16 tcgen05.mma (M=128,
//               N=NT, K=16) per chunk into one of two TMEM accumulators.
//   warps 4-11  epilogue: warp w reads TMEM lanes 32*(w%4) (its tile rows)
//               and one column half with tcgen05.ld, applies bias / LN fold /
//               SimpleGate / beta-gamma residual, writes a swizzled staging
//               tile, and one thread moves the tile out with TMA tensor stores
//               (the residual tile arrives the same way), or scatters
//               PixelShuffle(2)+skip directly.
// A 3-stage shared-memory ring and double-buffered accumulators overlap
// loads, MMAs and epilogues of consecutive tiles. Every wait is bounded.
//
// Replaces the reference's cudnnConvolutionForward + cudnnAddTensor pair
// (src/layers/conv2d.cu:94-150) and the separate LN / SimpleGate / SCA /
// scaled-add / pixel-shuffle / add kernels (src/kernels/nafnet_kernels.cu
// :54-208) around each 1x1 / 2x2 conv of a NAFBlock (src/models/nafnet.cu
// :146-255).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>

#include "kernels.h"
#include "launch.cuh"
#include "sm100.cuh"
#include "status.h"

namespace dnb {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

namespace {

constexpr int kRows = 128;
constexpr int kStages = 3;
constexpr int kKC = 64;                 // shared-memory footprint is sized for KC = 64
constexpr int kThreads = 480;
// The LayerNorm-folded kernels add warps 15-18: a second group of row
// statistics warps, so that each group handles every other ring stage.
constexpr int kThreadsLN = 608;
constexpr uint32_t kALbo = kRows * 16;  // 2 KB between K-adjacent core-matrix columns

struct GemmMaps {
    CUtensorMap a[kMaxSeg];
    CUtensorMap out;  // epilogue store (box EB x 128, swizzled)
    CUtensorMap res;  // residual load (same geometry as out)
};

// Named barrier of the eight epilogue warps.
__device__ __forceinline__ void epi_sync() { named_sync(1, 256); }

// Same barrier, returning the OR of `v` over the 256 epilogue threads (a
// uniform decision for all of them).
__device__ __forceinline__ bool epi_sync_or(bool v) { return named_sync_or(1, 256, v); }

// Source address of the 8 channels [k, k+8) of the 2x2/stride-2 patch of
// output pixel `pix` of image `img`.
__device__ __forceinline__ const __half* s2_src(const GemmParams& p, int img, int pix, int k) {
    const int tap = k / p.seg_c;
    const int c = k - tap * p.seg_c;
    const int y = pix / p.Wo;
    const int x = pix - y * p.Wo;
    const size_t spix = static_cast<size_t>(2 * y + (tap >> 1)) * (2 * p.Wo) + 2 * x + (tap & 1);
    return p.a[0] + img * p.a_img_stride + spix * p.seg_c + c;
}

// Epilogue staging geometry: boxes of EB columns x 128 rows, TMA-swizzled
// with a span of EB*2 bytes (32 / 64 / 128).
template <int OUTC>
struct Staging {
    static constexpr int EB = OUTC < 64 ? OUTC : 64;
    static constexpr int kBoxes = OUTC / EB;
    static constexpr int kRowBytes = EB * 2;
    static constexpr int kBoxBytes = kRows * kRowBytes;
    static constexpr int kBytes = kBoxes * kBoxBytes;
    // Byte offset of 16-byte chunk `j` (8 columns) of row r.
    __device__ static __forceinline__ uint32_t off(int r, int j) {
        const int box = j / (EB / 8);
        const int jj = j - box * (EB / 8);
        int sw;
        if (EB == 64) sw = r & 7;
        else if (EB == 32) sw = (r >> 1) & 3;
        else sw = (r >> 2) & 1;
        return box * kBoxBytes + r * kRowBytes + ((jj ^ sw) << 4);
    }
};

// Dynamic shared memory of one instantiation: the stage ring, the epilogue
// staging tile (none for the PixelShuffle scatter, which stores directly)
// and the parameter vectors it uses.
template <int PRO, int EPI, int NT, int AMODE = kARows>
struct SmemPlan {
    // CTA pairs: 4 stages of A (128 rows) + half of the B tile.
    static constexpr int kSt = AMODE == kARowsPair ? 4 : kStages;
    static constexpr int kStage = kRows * kKC * 2 + (AMODE == kARowsPair ? NT / 2 : NT) * kKC * 2;
    static constexpr int kOutCols = (EPI == kEpiGate) ? NT / 2 : NT;
    // The row-tiled shuffle stages both fine rows of its tile: 2 x 256 pixels x NT/4 channels.
    // At NT = 128 two such tiles alternate, so that the next tile's skip
    // loads while the current one is finished.
    static constexpr int kStgBytes = (EPI == kEpiShuffleAdd) ? 0
                                     : (EPI == kEpiShuffleRows) ? (NT <= 128 ? 2 : 1) * 256 * NT
                                                                : Staging<kOutCols>::kBytes;
    static int param_floats(const GemmParams& p) {
        return p.n_tiles * NT * (PRO == kProLayerNorm ? 2 : 1) + (EPI == kEpiResidual ? p.n_out : 0) +
               (PRO == kProScale ? p.K : 0);
    }
    static int bytes(const GemmParams& p) { return 1024 + kSt * kStage + kStgBytes + param_floats(p) * 4; }
};

template <int PRO, int EPI, int AMODE, int NT>
__global__ void __launch_bounds__(PRO == kProLayerNorm ? kThreadsLN : kThreads, 1)
    gemm_ws_kernel(const __grid_constant__ GemmParams p, const __grid_constant__ GemmMaps maps) {
    constexpr bool kLN = (PRO == kProLayerNorm);
    constexpr bool kWriteA = (PRO == kProScale) || (AMODE == kAS2x2);  // MMA waits for the transform
    // CTA pairs (kARowsPair): a tile is 256 rows; CTA `rank` of the pair owns
    // rows [128 rank, 128 rank + 128) and loads its A rows and B rows
    // [NT/2 rank, NT/2 rank + NT/2) into the same shared-memory offsets as its
    // peer; the even CTA issues the M = 256 MMAs for both, the odd CTA's MMA
    // thread forwards its stages' arrival to it.
    constexpr bool kPair = (AMODE == kARowsPair);
    using Plan = SmemPlan<PRO, EPI, NT, AMODE>;
    constexpr int kSt = Plan::kSt;
    constexpr uint32_t kAccCols = NT < 32 ? 32 : NT;
    constexpr uint32_t kCols = 2 * kAccCols;  // two accumulators
    constexpr int kOutCols = (EPI == kEpiGate) ? NT / 2 : NT;
    using Stg = Staging<kOutCols>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // Swizzled TMA staging needs 1024-byte alignment: align by hand (the
    // launch reserves 1 KB of slack).
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    __shared__ uint64_t bar_raw[kSt], bar_full[kSt], bar_empty[kSt], bar_peer[kSt], bar_done;
    __shared__ uint64_t bar_acc_full[2], bar_acc_empty[2], bar_st_full[2], bar_st_empty[2], bar_res, bar_skip[2];
    __shared__ float2 s_stats[2][kRows];  // LN (mean, rstd) per tile row, double-buffered
    __shared__ float2 s_part[2][kRows];   // LN: second statistics group's (sum, sum of squares) per tile row
    __shared__ uint64_t bar_part[2], bar_pfree[2];
    __shared__ uint32_t tslot;
    __shared__ volatile int s_abort;

    const int KC = p.KC;
    const int nk = p.k_chunks;
    const uint32_t a_bytes = kRows * KC * 2;
    const uint32_t b_bytes = NT * KC * 2;
    const uint32_t b_sbo = static_cast<uint32_t>(KC / 8) * 128u;
    const uint32_t stage_bytes = Plan::kStage;
    const uint32_t a_swz = static_cast<uint32_t>(p.a_swz);
    // Byte offset of 16-byte chunk q (8 channels) of tile row r in an A stage.
    auto a_off = [a_swz](int r, int q) -> uint32_t {
        return a_swz ? sw_offset(r, q, a_swz) : static_cast<uint32_t>(q) * kALbo + r * 16;
    };
    uint8_t* stg = smem + kSt * stage_bytes;  // 1024-aligned: stage_bytes is a multiple of 1024
    float* s_bias = reinterpret_cast<float*>(stg + Plan::kStgBytes);
    float* s_c1 = s_bias + p.n_tiles * NT;                                   // LN fold only
    float* s_rsc = s_c1 + (kLN ? p.n_tiles * NT : 0);                        // residual only
    float* s_sca = s_rsc + (EPI == kEpiResidual ? p.n_out : 0);             // SCA scale of image 0
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    // Row-aligned tiles (2x2 stride-2 by TMA, staged shuffle): a tile is up to
    // 128 pixels of one output row, so that its A rows / output rows map to
    // contiguous pixel runs; otherwise 128 consecutive rows of M.
    constexpr bool kRowT = (AMODE == kAPairs) || (EPI == kEpiShuffleRows);
    const int xch = kRowT ? (p.Wo + kRows - 1) / kRows : 1;
    constexpr int kTileRows = kPair ? 2 * kRows : kRows;
    const int m_tiles = kRowT ? (p.M / p.Wo) * xch : (p.M + kTileRows - 1) / kTileRows;
    const uint32_t rank = kPair ? cluster_rank() : 0u;
    const int tile0 = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
    const int tstep = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
    const int n_tiles_total = m_tiles * p.n_tiles;
    const bool one_img = p.M <= p.hw;
    // m0: first row of the tile in M; rid / x0: output row and first column
    // (row-aligned tiles); nval: rows of the tile that exist.
    auto tgeo = [&](int tile, int& m0, int& rid, int& x0, int& nval) {
        const int tm = tile / p.n_tiles;
        if (kRowT) {
            rid = tm / xch;
            x0 = (tm - rid * xch) * kRows;
            m0 = rid * p.Wo + x0;
            nval = min(kRows, p.Wo - x0);
        } else {
            rid = 0;
            x0 = 0;
            m0 = tm * kTileRows + static_cast<int>(rank) * kRows;
            nval = min(kRows, p.M - m0);  // <= 0 for the odd CTA past the last row
        }
    };

    // The tensor maps this instantiation uses (the ones the launcher encoded).
    if (tid == 0) {
        if (AMODE != kAS2x2)
            for (int sgi = 0; sgi < (AMODE == kAPairs ? 1 : p.nseg); ++sgi) prefetch_tmap(&maps.a[sgi]);
        const bool out_map = (EPI == kEpiShuffleRows) || ((EPI != kEpiShuffleAdd) && (p.out_c % kOutCols == 0));
        if (out_map) prefetch_tmap(&maps.out);
        if (out_map && (EPI == kEpiResidual || EPI == kEpiShuffleRows)) prefetch_tmap(&maps.res);
    }
    // Parameter vectors -> shared memory (c2 of the LN fold lives in s_bias).
    constexpr int kNThr = kLN ? kThreadsLN : kThreads;
    for (int i = tid; i < p.n_tiles * NT; i += kNThr) {
        s_bias[i] = p.bias ? p.bias[i] : 0.f;
        if (kLN) s_c1[i] = p.ln_c1[i];
    }
    if (EPI == kEpiResidual)
        for (int i = tid; i < p.n_out; i += kNThr) s_rsc[i] = p.res_scale[i];
    if (warp == 0) {
        if (kPair) {
            tmem_alloc_pair(&tslot, kCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(&tslot, kCols);
            tmem_relinquish();
        }
    }
    if (tid == 0) {
        for (int s = 0; s < kSt; ++s) {
            mbar_init(&bar_raw[s], 2);  // the A and the B producer
            mbar_init(&bar_full[s], 4);
            mbar_init(&bar_empty[s], kLN ? 5 : 1);  // LN: MMA commit + 4 statistics warps
            mbar_init(&bar_peer[s], 1);             // pairs: the odd CTA's stage has landed
        }
        mbar_init(&bar_done, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bar_acc_full[b], 1);
            mbar_init(&bar_acc_empty[b], kPair ? 16 : 8);  // pairs: both CTAs' epilogue warps
            mbar_init(&bar_st_full[b], 4);
            mbar_init(&bar_st_empty[b], 8);
        }
        mbar_init(&bar_res, 1);
        mbar_init(&bar_skip[0], 1);
        mbar_init(&bar_skip[1], 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bar_part[b], 4);
            mbar_init(&bar_pfree[b], 4);
        }
        s_abort = 0;
        fence_mbar_init();
    }
    tc_fence_before();
    if (kPair)
        cluster_sync_all();  // both CTAs' barriers exist before either arrives on the other's
    else
        __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    pdl_trigger();  // only once this CTA holds its TMEM columns
    // Everything above touched only weights; activations (A, the residual,
    // the SCA scale) were written by earlier kernels.
    pdl_wait();
    if (PRO == kProScale && one_img) {
        for (int i = tid; i < p.K; i += kNThr) s_sca[i] = p.pro_scale[i];
        __syncthreads();
    }

    if (warp == 12 || warp == 14) {
        // ------------------------------ TMA producers -----------------------------
        // Warp 12 loads the A rows, warp 14 the B tile of each stage: one
        // issuing thread sustains about one copy per microsecond-scale copy
        // latency, so the two operands stream from separate threads.
        const bool is_b = (warp == 14);
        if (lane == 0) {
            int it = 0;
            for (int tile = tile0; tile < n_tiles_total && !s_abort; tile += tstep) {
                const int n_tile = tile % p.n_tiles;
                int m0, rid, x0, nval;
                tgeo(tile, m0, rid, x0, nval);
                for (int j = 0; j < nk; ++j, ++it) {
                    const int s = it % kSt;
                    const uint32_t ph = (it / kSt) & 1;
                    if (!wait_or_abort(&bar_empty[s], ph ^ 1, &s_abort, p.err, 0x20)) break;
                    uint8_t* sa = smem + s * stage_bytes;
                    uint8_t* sb = sa + kRows * kKC * 2;
                    if (is_b) {
                        // Pairs: this CTA's half of the B tile (its first NT/2 rows are
                        // the first half of the tile image).
                        const uint32_t bb = kPair ? b_bytes / 2 : b_bytes;
                        mbar_arrive_expect_tx(&bar_raw[s], bb);
                        bulk_g2s(sb, p.bpack + (static_cast<size_t>(n_tile) * nk + j) * b_bytes + rank * bb, bb,
                                 &bar_raw[s]);
                        continue;
                    }
                    mbar_arrive_expect_tx(&bar_raw[s], AMODE == kAS2x2 ? 0u : a_bytes);
                    if (AMODE == kAPairs) {
                        // Input row 2*rid + ky as pixel pairs: k = (2 ky + kx) C + c.
                        const int k0 = j * KC;
                        const int ky = k0 / (2 * p.seg_c);
                        tma_load_3d(sa, &maps.a[0], k0 - ky * 2 * p.seg_c, x0, 2 * rid + ky, &bar_raw[s]);
                    } else if (AMODE != kAS2x2) {
                        const int k0 = j * KC;
                        if (a_swz) {
                            // One KC-wide swizzled box (KC <= segment width).
                            const int seg = k0 / p.seg_c;
                            const bool in = k0 < p.K;
                            tma_load_2d(sa, &maps.a[in ? seg : 0], in ? k0 - seg * p.seg_c : p.seg_c, m0, &bar_raw[s]);
                        } else {
                            for (int q = 0; q < KC / 8; ++q) {
                                const int k = k0 + q * 8;
                                const int seg = k < p.K ? k / p.seg_c : 0;
                                const int kl = k < p.K ? k - seg * p.seg_c : p.seg_c;  // OOB -> zero fill
                                tma_load_2d(sa + q * kALbo, &maps.a[seg], kl, m0, &bar_raw[s]);
                            }
                        }
                    }
                }
            }
            // Pairs: the even CTA's MMA commits arrive on this CTA's stage
            // barriers; before the CTA may exit, every issued stage must have
            // been released (so no arrive lands after it).
            if (kPair && !is_b && !s_abort)
                for (int k = max(0, it - kSt); k < it; ++k)
                    if (!wait_or_abort(&bar_empty[k % kSt], (k / kSt) & 1, &s_abort, p.err, 0x2c)) break;
        }
    } else if (warp == 13) {
        // ------------------------------ MMA issuer --------------------------------
        if (lane == 0 && kPair && rank == 1) {
            // The odd CTA of a pair: forward each stage's arrival in this CTA's
            // shared memory to the even CTA, whose thread issues the MMAs.
            int s = 0;
            uint32_t ph = 0;
            for (int tile = tile0; tile < n_tiles_total && !s_abort; tile += tstep) {
                bool ok = true;
                for (int j = 0; j < nk; ++j) {
                    if (!wait_or_abort(kWriteA ? &bar_full[s] : &bar_raw[s], ph, &s_abort, p.err, 0x2d)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_remote(peer_addr(&bar_peer[s], 0));
                    if (++s == kSt) {
                        s = 0;
                        ph ^= 1;
                    }
                }
                if (!ok) break;
            }
        } else if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(kPair ? 2 * kRows : kRows, NT);
            // The issuing thread is on the critical path of every stage: the
            // descriptors of stage 0 are built once, and each MMA only adds a
            // stage offset and a K-step offset (16-byte units) to them.
            const uint32_t sm0 = smem_u32(smem);
            const uint64_t ad0 = a_swz ? sdesc_kmajor_sw(sm0, a_swz) : sdesc_kmajor(sm0, kALbo, 128);
            const uint64_t bd0 = sdesc_kmajor(sm0 + kRows * kKC * 2, 128, b_sbo);
            const uint32_t a_kstep = a_swz ? 2u : (2u * kALbo) >> 4;  // one K=16 step
            const int nks = KC / 16;
            int s = 0, t = 0;
            uint32_t ph = 0;
            for (int tile = tile0; tile < n_tiles_total && !s_abort; tile += tstep, ++t) {
                const int b = t & 1;
                if (!wait_or_abort(&bar_acc_empty[b], ((t >> 1) & 1) ^ 1, &s_abort, p.err, 0x21)) break;
                tc_fence_after();
                const uint32_t acc = tmem + b * kAccCols;
                bool ok = true;
                for (int j = 0; j < nk; ++j) {
                    if (!wait_or_abort(kWriteA ? &bar_full[s] : &bar_raw[s], ph, &s_abort, p.err, 0x22) ||
                        (kPair && !wait_or_abort(&bar_peer[s], ph, &s_abort, p.err, 0x2e))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t so = static_cast<uint64_t>(s) * (stage_bytes >> 4);
                    const uint64_t ad = ad0 + so, bd = bd0 + so;
#pragma unroll
                    for (int k = 0; k < kKC / 16; ++k) {
                        if (k < nks) {
                            if (kPair)
                                mma_f16_pair(acc, ad + k * a_kstep, bd + 16 * k, idesc, (j > 0 || k > 0) ? 1u : 0u);
                            else
                                mma_f16(acc, ad + k * a_kstep, bd + 16 * k, idesc, (j > 0 || k > 0) ? 1u : 0u);
                        }
                    }
                    if (kPair)
                        mma_commit_pair(&bar_empty[s]);  // both CTAs' stage s
                    else
                        mma_commit(&bar_empty[s]);
                    if (++s == kSt) {
                        s = 0;
                        ph ^= 1;
                    }
                }
                if (!ok) break;
                if (kPair)
                    mma_commit_pair(&bar_acc_full[b]);
                else
                    mma_commit(&bar_acc_full[b]);
            }
        }
    } else if (warp < 4 || warp >= 15) {
        // ------------------------------ transform ---------------------------------
        // LN: statistics group g (warps 0-3, or 15-18) takes the ring stages
        // it with it % 2 == g; group 1 hands its partial sums of each tile to
        // group 0 through s_part.
        const int g = warp >= 15 ? 1 : 0;
        if (kLN || kWriteA) {
            const int r = g ? tid - 15 * 32 : tid;  // tile row
            int it = 0, t = 0;
            int s2_prev = -1;  // 2x2 gather: stage whose copies are still in flight
            for (int tile = tile0; tile < n_tiles_total && !s_abort; tile += tstep, ++t) {
                int m0, rid, tx0, nval;
                tgeo(tile, m0, rid, tx0, nval);
                const int row = m0 + r;
                const bool row_ok = row < p.M;
                const int img = row_ok ? row / p.hw : 0;
                const int pix = row - img * p.hw;
                float s1 = 0.f, s2 = 0.f;
                bool ok = true;
                for (int j = 0; j < nk; ++j, ++it) {
                    if (kLN && (it & 1) != g) continue;  // the other group's stage
                    const int s = it % kSt;
                    const uint32_t ph = (it / kSt) & 1;
                    if (!wait_or_abort(&bar_raw[s], ph, &s_abort, p.err, 0x23)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sa = smem + s * stage_bytes;
                    if (kLN) {
                        // Row sums and sums of squares. The stage is released as
                        // soon as its values are in registers (the arrive orders
                        // the reads before the producer's next write).
                        const int nq = min(KC, p.K - j * KC) >> 3;
                        uint4 v[8];
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            if (q < nq) v[q] = *reinterpret_cast<const uint4*>(sa + a_off(r, q));
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&bar_empty[s]);
                        const float2 one = make_float2(1.f, 1.f);
                        float2 a1[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
                        float2 a2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            if (q < nq) {
                                const uint32_t w[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
                                for (int i = 0; i < 4; ++i) {
                                    const float2 x = unpack_half2(w[i]);
                                    a1[i & 1] = ffma2(x, one, a1[i & 1]);
                                    a2[i & 1] = ffma2(x, x, a2[i & 1]);
                                }
                            }
                        }
                        s1 += (a1[0].x + a1[0].y) + (a1[1].x + a1[1].y);
                        s2 += (a2[0].x + a2[0].y) + (a2[1].x + a2[1].y);
                    } else if (AMODE == kAS2x2) {
                        // Gather this stage's patch rows with cp.async (zero fill
                        // outside), then release the previous stage once its copies
                        // have landed: one stage of gathers stays in flight.
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            const int k = j * KC + q * 8;
                            if (q * 8 < KC) {
                                const bool valid = row_ok && k < p.K;
                                cp_async16_zfill(sa + a_off(r, q), valid ? s2_src(p, img, pix, k) : p.a[0], valid);
                            }
                        }
                        cp_async_commit();
                        if (s2_prev >= 0) {
                            cp_async_wait<1>();
                            fence_async_smem();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&bar_full[s2_prev]);
                        }
                        s2_prev = s;
                    } else {  // SCA scale in place
                        if (row_ok) {
                            const float* sc = one_img ? s_sca : p.pro_scale + static_cast<size_t>(img) * p.K;
                            for (int q = 0; q < KC / 8; ++q) {
                                const int k = j * KC + q * 8;
                                if (k >= p.K) break;
                                uint4* ptr = reinterpret_cast<uint4*>(sa + a_off(r, q));
                                float f[8];
                                h8_to_f(*ptr, f);
#pragma unroll
                                for (int i = 0; i < 8; ++i) f[i] *= sc[k + i];
                                *ptr = f_to_h8(f);
                            }
                        }
                        fence_async_smem();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&bar_full[s]);
                    }
                }
                if (!ok) break;
                if (kLN) {
                    const int sb = t & 1;
                    const uint32_t pp = (t >> 1) & 1;
                    if (g == 1) {
                        // Hand the partial sums over (the slot of tile t - 2 must
                        // have been read first).
                        if (!wait_or_abort(&bar_pfree[sb], pp ^ 1, &s_abort, p.err, 0x2a)) break;
                        s_part[sb][r] = make_float2(s1, s2);
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&bar_part[sb]);
                        continue;
                    }
                    if (!wait_or_abort(&bar_part[sb], pp, &s_abort, p.err, 0x2b)) break;
                    const float2 o = s_part[sb][r];
                    s1 += o.x;
                    s2 += o.y;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bar_pfree[sb]);
                    if (!wait_or_abort(&bar_st_empty[sb], ((t >> 1) & 1) ^ 1, &s_abort, p.err, 0x25)) break;
                    const float inv = 1.0f / static_cast<float>(p.K);
                    const float dm = s1 * inv;
                    const float var = fmaxf(s2 * inv - dm * dm, 0.f);
                    s_stats[sb][r] = make_float2(dm, rsqrtf(var + 1e-6f));
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bar_st_full[sb]);
                }
            }
            if (AMODE == kAS2x2) {
                // Release the last gathered stage (and let every copy land).
                cp_async_wait<0>();
                fence_async_smem();
                __syncwarp();
                if (s2_prev >= 0 && lane == 0 && !s_abort) mbar_arrive(&bar_full[s2_prev]);
            }
        }
    } else {
        // ------------------------------ epilogue ----------------------------------
        // Warps 4-11: warp w reads TMEM lanes 32*(w%4).. (its tile rows) and
        // column half (w-4)/4 of the tile (all columns if the tile is narrow).
        const int wq = warp & 3;                 // TMEM lane quarter of this warp
        const int r = wq * 32 + lane;            // tile row == TMEM lane
        const int ch = (warp - 4) >> 2;          // column group
        const bool leader = (tid == 128);
        // The accumulator is drained: pairs count both CTAs' epilogue warps on
        // the even CTA's barrier.
        auto release_acc = [&](int b) {
            if (kPair && rank == 1)
                mbar_arrive_remote(peer_addr(&bar_acc_empty[b], 0));
            else
                mbar_arrive(&bar_acc_empty[b]);
        };
        // [lo, hi) of a span of `cols` columns for this warp's group (spans
        // narrower than 32 stay with group 0)
        auto span = [ch](int cols, int& lo, int& hi) {
            if (cols >= 32) {
                lo = ch * (cols / 2);
                hi = lo + cols / 2;
            } else {
                lo = 0;
                hi = ch == 0 ? cols : 0;
            }
        };
        const bool tma_epi = (EPI == kEpiShuffleRows) || ((EPI != kEpiShuffleAdd) && (p.out_c % kOutCols == 0));
        int pf_slot = -1;        // staged shuffle: slot of a skip prefetch not yet waited for (leader)
        uint32_t pf_par = 0;
        int t = 0;
        for (int tile = tile0; tile < n_tiles_total; tile += tstep, ++t) {
            const int b = t & 1;
            bool got = wait_or_abort(&bar_acc_full[b], (t >> 1) & 1, &s_abort, p.err, 0x24);
            if (kLN && got) got = wait_or_abort(&bar_st_full[b], (t >> 1) & 1, &s_abort, p.err, 0x26);
            // previous tile's store has read the staging (the double-buffered
            // shuffle waits for its other buffer instead, before its prefetch)
            if (tma_epi && leader && !(EPI == kEpiShuffleRows && NT <= 128)) bulk_wait_read0();
            // Uniform exit decision; also the "staging is free again" barrier.
            if (epi_sync_or(!got || s_abort)) break;
            tc_fence_after();
            const int n_tile = tile % p.n_tiles;
            int m0, rid, x0, nval;
            tgeo(tile, m0, rid, x0, nval);
            const int row = m0 + r;
            const bool row_ok = r < nval;
            const int img = row_ok ? row / p.hw : 0;
            const int pix = row - img * p.hw;
            const uint32_t lane_base = tmem + b * kAccCols + (static_cast<uint32_t>(wq * 32) << 16);
            float mean = 0.f, rstd = 1.f;
            if (kLN) {
                const float2 st = s_stats[b][r];
                mean = st.x;
                rstd = st.y;
                __syncwarp();
                if (lane == 0) mbar_arrive(&bar_st_empty[b]);
            }
            const int col0 = n_tile * kOutCols;
            if (EPI == kEpiResidual && tma_epi) {
                if (leader) {
                    mbar_arrive_expect_tx(&bar_res, Stg::kBytes);
                    for (int bx = 0; bx < Stg::kBoxes; ++bx)
                        tma_load_2d(stg + bx * Stg::kBoxBytes, &maps.res, col0 + bx * Stg::EB, m0, &bar_res);
                }
                wait_or_abort(&bar_res, t & 1, &s_abort, p.err, 0x27);
            }
            if (EPI == kEpiShuffleRows) {
                // PixelShuffle(2) + skip through the staging tile: column n =
                // ij * cout + ch of coarse pixel (rid, x0 + r) lands at fine
                // pixel (2 rid + ij/2, 2 (x0 + r) + ij%2). The tile's outputs are
                // two contiguous runs of 256 fine pixels (rows 2 rid, 2 rid + 1):
                // the skip of both arrives by TMA into the staging tile, each
                // thread adds its values in place, and TMA stores the two rows
                // (columns past the image are clipped by the tensor map). With
                // two staging tiles (NT = 128), tile t uses tile t % 2, and the
                // skip of the next tile is requested as soon as the stores of
                // tile t - 1 have read its buffer.
                constexpr int kCout = NT / 4;
                constexpr int kRowBytes = kCout * 2;
                constexpr int kFineRow = 256 * kRowBytes;
                constexpr bool kDbl = NT <= 128;
                uint8_t* sb = stg + (kDbl ? (t & 1) * 2 * kFineRow : 0);
                auto skip_load = [&](int tl, uint8_t* dst, uint64_t* bar) {
                    int tm0, trid, tx0, tnv;
                    tgeo(tl, tm0, trid, tx0, tnv);
                    mbar_arrive_expect_tx(bar, 2 * kFineRow);
                    tma_load_3d(dst, &maps.res, 0, 2 * tx0, 2 * trid, bar);
                    tma_load_3d(dst + kFineRow, &maps.res, 0, 2 * tx0, 2 * trid + 1, bar);
                };
                if (leader && (!kDbl || t == 0)) skip_load(tile, sb, &bar_skip[kDbl ? (t & 1) : 0]);
                const int sk_slot = kDbl ? (t & 1) : 0;
                const uint32_t sk_par = kDbl ? ((t >> 1) & 1) : (t & 1);
                wait_or_abort(&bar_skip[sk_slot], sk_par, &s_abort, p.err, 0x28);
                pf_slot = -1;
                int c_lo, c_hi;
                span(NT, c_lo, c_hi);
#pragma unroll 1
                for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
                    float va[16];
                    tmem_ld16(lane_base + c0, va);
                    tmem_ld_wait();
                    if (!row_ok) continue;
#pragma unroll
                    for (int g = 0; g < 2; ++g) {
                        const int n = c0 + 8 * g;
                        const int ij = n / kCout, ch = n - ij * kCout;
                        uint8_t* sp = sb + (ij >> 1) * kFineRow + sw_offset(2 * r + (ij & 1), ch >> 3, kRowBytes);
                        float f[8], rr[8];
                        h8_to_f(*reinterpret_cast<const uint4*>(sp), rr);
#pragma unroll
                        for (int i = 0; i < 8; ++i) f[i] = va[8 * g + i] + s_bias[n + i] + rr[i];
                        *reinterpret_cast<uint4*>(sp) = f_to_h8(f);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) release_acc(b);
                fence_async_smem();
                epi_sync();
                if (leader) {
                    tma_store_3d(&maps.out, 0, 2 * x0, 2 * rid, sb);
                    tma_store_3d(&maps.out, 0, 2 * x0, 2 * rid + 1, sb + kFineRow);
                    bulk_commit();
                    const int next = tile + static_cast<int>(gridDim.x);
                    if (kDbl && next < n_tiles_total) {
                        // The other buffer was last read by tile t - 1's stores.
                        bulk_wait_read1();
                        skip_load(next, stg + ((t + 1) & 1) * 2 * kFineRow, &bar_skip[(t + 1) & 1]);
                        pf_slot = (t + 1) & 1;
                        pf_par = static_cast<uint32_t>(((t + 1) >> 1) & 1);
                    }
                }
                continue;
            }
            if (EPI == kEpiShuffleAdd) {
                // PixelShuffle(2) scatter + skip: column n = ij * cout + ch of input
                // pixel (y, x) lands at output pixel (2y + ij/2, 2x + ij%2),
                // channel ch. The skip vectors of 8 column groups are loaded
                // before any is used (one memory latency per 64 columns).
                int c_lo, c_hi;
                span(kOutCols, c_lo, c_hi);
                const int cout = p.out_c;
                const int y = pix / p.Wo;
                const int x = pix - y * p.Wo;
                auto soff = [&](int n) -> size_t {
                    const int ij = n / cout;
                    const int ch = n - ij * cout;
                    const size_t opix = (static_cast<size_t>(img) * (2 * p.Ho) + 2 * y + (ij >> 1)) * (2 * p.Wo) +
                                        2 * x + (ij & 1);
                    return opix * cout + ch;
                };
#pragma unroll 1
                for (int cb = c_lo; cb < c_hi; cb += 64) {
                    uint4 sk[8];
#pragma unroll
                    for (int g = 0; g < 8; ++g) {
                        const int c = cb + 8 * g;
                        sk[g] = make_uint4(0, 0, 0, 0);
                        if (row_ok && c < c_hi && col0 + c < p.n_out)
                            sk[g] = __ldg(reinterpret_cast<const uint4*>(p.skip + soff(n_tile * NT + c)));
                    }
#pragma unroll
                    for (int h = 0; h < 4; ++h) {
                        const int c0 = cb + 16 * h;
                        if (c0 >= c_hi) break;  // uniform across the warp
                        float va[16];
                        tmem_ld16(lane_base + c0, va);
                        tmem_ld_wait();
                        if (!row_ok) continue;
#pragma unroll
                        for (int g = 0; g < 2; ++g) {
                            const int n = n_tile * NT + c0 + 8 * g;
                            if (col0 + c0 + 8 * g >= p.n_out) break;
                            float f[8], rr[8];
                            h8_to_f(sk[2 * h + g], rr);
#pragma unroll
                            for (int i = 0; i < 8; ++i) f[i] = va[8 * g + i] + s_bias[n + i] + rr[i];
                            *reinterpret_cast<uint4*>(p.out + soff(n)) = f_to_h8(f);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) release_acc(b);
                continue;
            }
            if (!tma_epi) {
                // Direct per-row stores from registers (outputs narrower than a
                // staging box): per 64 columns the
                // residual vectors are loaded before any is used; the LN fold
                // and the gate run in packed fp32 as in the staged path.
                int c_lo, c_hi;
                span(kOutCols, c_lo, c_hi);
                const float2 one2 = make_float2(1.f, 1.f);
                const float2 rs2 = make_float2(rstd, rstd);
                const float2 nm2 = make_float2(-rstd * mean, -rstd * mean);
                auto fold = [&](const float* acc, int n, float2 (&y)[4]) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float2 bb = make_float2(s_bias[n + 2 * i], s_bias[n + 2 * i + 1]);
                        if (kLN)
                            y[i] = ffma2(rs2, make_float2(acc[2 * i], acc[2 * i + 1]),
                                         ffma2(nm2, make_float2(s_c1[n + 2 * i], s_c1[n + 2 * i + 1]), bb));
                        else
                            y[i] = ffma2(make_float2(acc[2 * i], acc[2 * i + 1]), one2, bb);
                    }
                };
                const size_t rowoff = static_cast<size_t>(row) * p.out_c;
#pragma unroll 1
                for (int cb = c_lo; cb < c_hi; cb += 64) {
                    uint4 rv[8];
                    if (EPI == kEpiResidual) {
#pragma unroll
                        for (int g = 0; g < 8; ++g) {
                            const int o = col0 + cb + 8 * g;
                            rv[g] = (row_ok && cb + 8 * g < c_hi && o < p.n_out)
                                        ? *reinterpret_cast<const uint4*>(p.res + rowoff + o)
                                        : make_uint4(0u, 0u, 0u, 0u);
                        }
                    }
#pragma unroll
                    for (int h = 0; h < 4; ++h) {
                        const int c0 = cb + 16 * h;
                        if (c0 >= c_hi) break;  // uniform across the warp
                        float va[16], vb[16];
                        tmem_ld16(lane_base + c0, va);
                        if (EPI == kEpiGate) tmem_ld16(lane_base + NT / 2 + c0, vb);
                        tmem_ld_wait();
                        if (!row_ok) continue;
#pragma unroll
                        for (int g = 0; g < 2; ++g) {
                            const int n = n_tile * NT + c0 + 8 * g;
                            const int o = col0 + c0 + 8 * g;
                            if (o >= p.n_out) break;
                            float2 y[4];
                            fold(va + 8 * g, n, y);
                            if (EPI == kEpiGate) {
                                float2 y2[4];
                                fold(vb + 8 * g, n + NT / 2, y2);
#pragma unroll
                                for (int i = 0; i < 4; ++i) y[i] = ffma2(y[i], y2[i], make_float2(0.f, 0.f));
                            }
                            if (EPI == kEpiStore && p.relu) {
#pragma unroll
                                for (int i = 0; i < 4; ++i) y[i] = make_float2(fmaxf(y[i].x, 0.f), fmaxf(y[i].y, 0.f));
                            }
                            if (EPI == kEpiResidual) {
                                const uint4 rr = rv[2 * h + g];
                                const uint32_t rw[4] = {rr.x, rr.y, rr.z, rr.w};
#pragma unroll
                                for (int i = 0; i < 4; ++i)
                                    y[i] = ffma2(make_float2(s_rsc[o + 2 * i], s_rsc[o + 2 * i + 1]), y[i],
                                                 unpack_half2(rw[i]));
                            }
                            *reinterpret_cast<uint4*>(p.out + rowoff + o) =
                                make_uint4(pack_half2(y[0].x, y[0].y), pack_half2(y[1].x, y[1].y),
                                           pack_half2(y[2].x, y[2].y), pack_half2(y[3].x, y[3].y));
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) release_acc(b);
                continue;
            }
            // Swizzled staging tile -> TMA tensor store. Per 8 columns:
            // LN fold  y = rstd * acc + (c2 - rstd * mean * c1), else y = acc + bias,
            // in packed f32x2 arithmetic with float4 parameter loads.
            const float2 one2 = make_float2(1.f, 1.f);
            const float2 rs2 = make_float2(rstd, rstd);
            const float2 nm2 = make_float2(-rstd * mean, -rstd * mean);
            // 8 columns starting at n: acc (8 values) -> bias/LN-folded values
            auto fold8 = [&](const float* acc, int n, float2 (&y)[4]) {
                const float4 b0 = *reinterpret_cast<const float4*>(s_bias + n);
                const float4 b1 = *reinterpret_cast<const float4*>(s_bias + n + 4);
                const float2 bb[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w), make_float2(b1.x, b1.y),
                                      make_float2(b1.z, b1.w)};
                if (kLN) {
                    const float4 k0 = *reinterpret_cast<const float4*>(s_c1 + n);
                    const float4 k1 = *reinterpret_cast<const float4*>(s_c1 + n + 4);
                    const float2 cc[4] = {make_float2(k0.x, k0.y), make_float2(k0.z, k0.w), make_float2(k1.x, k1.y),
                                          make_float2(k1.z, k1.w)};
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        y[i] = ffma2(rs2, make_float2(acc[2 * i], acc[2 * i + 1]), ffma2(nm2, cc[i], bb[i]));
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) y[i] = ffma2(make_float2(acc[2 * i], acc[2 * i + 1]), one2, bb[i]);
                }
            };
            if (EPI == kEpiGate) {
                constexpr int kHalf = NT / 2;
                int c_lo, c_hi;
                span(kHalf, c_lo, c_hi);
#pragma unroll 1
                for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
                    float va[16], vb[16];
                    tmem_ld16(lane_base + c0, va);
                    tmem_ld16(lane_base + kHalf + c0, vb);
                    tmem_ld_wait();
                    const int n = n_tile * NT + c0;
#pragma unroll
                    for (int g = 0; g < 2; ++g) {
                        float2 x1[4], x2[4];
                        fold8(va + 8 * g, n + 8 * g, x1);
                        fold8(vb + 8 * g, n + kHalf + 8 * g, x2);
                        uint4 o;
                        const float2 z = make_float2(0.f, 0.f);
                        const float2 p0 = ffma2(x1[0], x2[0], z), p1 = ffma2(x1[1], x2[1], z);
                        const float2 p2 = ffma2(x1[2], x2[2], z), p3 = ffma2(x1[3], x2[3], z);
                        o.x = pack_half2(p0.x, p0.y);
                        o.y = pack_half2(p1.x, p1.y);
                        o.z = pack_half2(p2.x, p2.y);
                        o.w = pack_half2(p3.x, p3.y);
                        *reinterpret_cast<uint4*>(stg + Stg::off(r, (c0 >> 3) + g)) = o;
                    }
                }
            } else {
                constexpr int kStep = NT >= 64 ? 32 : 16;
                int c_lo, c_hi;
                span(NT, c_lo, c_hi);
#pragma unroll 1
                for (int c0 = c_lo; c0 < c_hi; c0 += kStep) {
                    float va[32];
                    tmem_ld16(lane_base + c0, *reinterpret_cast<float(*)[16]>(va));
                    if (kStep == 32) tmem_ld16(lane_base + c0 + 16, *reinterpret_cast<float(*)[16]>(va + 16));
                    tmem_ld_wait();
                    const int n = n_tile * NT + c0;
#pragma unroll
                    for (int g = 0; g < kStep / 8; ++g) {
                        float2 y[4];
                        fold8(va + 8 * g, n + 8 * g, y);
                        if (EPI == kEpiStore && p.relu) {
#pragma unroll
                            for (int i = 0; i < 4; ++i) y[i] = make_float2(fmaxf(y[i].x, 0.f), fmaxf(y[i].y, 0.f));
                        }
                        uint4* sp = reinterpret_cast<uint4*>(stg + Stg::off(r, (c0 >> 3) + g));
                        if (EPI == kEpiResidual) {
                            const uint4 rv = *sp;
                            const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
                            const int o = col0 + c0 + 8 * g;
                            float2 sc[4];
                            if (o + 8 <= p.n_out) {
                                const float4 q0 = *reinterpret_cast<const float4*>(s_rsc + o);
                                const float4 q1 = *reinterpret_cast<const float4*>(s_rsc + o + 4);
                                sc[0] = make_float2(q0.x, q0.y);
                                sc[1] = make_float2(q0.z, q0.w);
                                sc[2] = make_float2(q1.x, q1.y);
                                sc[3] = make_float2(q1.z, q1.w);
                            } else {
#pragma unroll
                                for (int i = 0; i < 4; ++i)
                                    sc[i] = make_float2(s_rsc[min(o + 2 * i, p.n_out - 1)],
                                                        s_rsc[min(o + 2 * i + 1, p.n_out - 1)]);
                            }
#pragma unroll
                            for (int i = 0; i < 4; ++i) y[i] = ffma2(sc[i], y[i], unpack_half2(rw[i]));
                        }
                        *sp = make_uint4(pack_half2(y[0].x, y[0].y), pack_half2(y[1].x, y[1].y),
                                         pack_half2(y[2].x, y[2].y), pack_half2(y[3].x, y[3].y));
                    }
                }
            }
            // TMEM of this accumulator is no longer needed.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) release_acc(b);
            fence_async_smem();
            epi_sync();
            if (leader && nval > 0) {  // (the odd CTA of a pair can lie wholly past the last row)
                for (int bx = 0; bx < Stg::kBoxes; ++bx) {
                    if (kRowT)
                        tma_store_3d(&maps.out, col0 + bx * Stg::EB, x0, rid, stg + bx * Stg::kBoxBytes);
                    else
                        tma_store_2d(&maps.out, col0 + bx * Stg::EB, m0, stg + bx * Stg::kBoxBytes);
                }
                bulk_commit();
            }
        }
        // The last store has read the staging tile (its writes complete with
        // the grid, before any dependent grid passes its wait).
        if (leader) bulk_wait_read0();
        // After an abort, a skip prefetch may still be landing in shared memory.
        if (EPI == kEpiShuffleRows && leader && pf_slot >= 0) mbar_wait(&bar_skip[pf_slot], pf_par, 5000000ull);
    }

    __syncthreads();
    if (s_abort && tid == 0) {
        // Let in-flight copies and MMAs land before the CTA's memory is released.
        for (int s = 0; s < kSt; ++s) {
            mbar_wait(&bar_raw[s], 0, 5000000ull);
            mbar_wait(&bar_empty[s], 0, 5000000ull);
        }
    }
    if (kPair && tid == 0) {
        // Neither CTA of a pair leaves (or frees its TMEM) before the other
        // is done with the MMAs that read its shared memory and with its
        // arrives on the other's barriers.
        mbar_arrive_remote(peer_addr(&bar_done, rank ^ 1u));
        if (!mbar_wait(&bar_done, 0)) report_error(p.err, 0x2f, kErrMbarTimeout);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        if (kPair)
            tmem_dealloc_pair(tmem, kCols);
        else
            tmem_dealloc(tmem, kCols);
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() { return tensor_map_encoder(); }

// 2-D map over a [rows][cols] fp16 matrix with row stride `ld` elements and a
// box of `box_cols` columns x 128 rows.
int make_map(CUtensorMap* m, const void* base, long long rows, int cols, long long ld, int box_cols,
             CUtensorMapSwizzle swz) {
    auto fn = encode_fn();
    if (!fn) return dn_fail(DN_ERR_CUDA, "gemm: cuTensorMapEncodeTiled unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * 2) % 16)
        return dn_fail(DN_ERR_INVALID_ARG, "gemm: operand must be 16-byte aligned");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), kRows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return dn_fail_str(DN_ERR_CUDA, "gemm: cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
    return DN_OK;
}

// 3-D map over rows of `width` pixels of `ch` fp16 channels ([rows][width][ch],
// contiguous) with a box of box_ch x box_w x 1 (pixels past `width` and rows
// past `rows` read as zero and are not written).
int make_map3(CUtensorMap* m, const void* base, long long rows, int width, int ch, int box_ch, int box_w,
              CUtensorMapSwizzle swz) {
    auto fn = encode_fn();
    if (!fn) return dn_fail(DN_ERR_CUDA, "gemm: cuTensorMapEncodeTiled unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (ch * 2) % 16)
        return dn_fail(DN_ERR_INVALID_ARG, "gemm: operand must be 16-byte aligned");
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(ch), static_cast<cuuint64_t>(width),
                                static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(ch) * 2, static_cast<cuuint64_t>(width) * ch * 2};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(box_ch), static_cast<cuuint32_t>(box_w), 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return dn_fail_str(DN_ERR_CUDA, "gemm: cuTensorMapEncodeTiled (3-D) failed (" + std::to_string(r) + ")");
    return DN_OK;
}

CUtensorMapSwizzle swizzle_for(int row_bytes) {
    return row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
           : row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                             : CU_TENSOR_MAP_SWIZZLE_32B;
}

int num_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// Kernels launched by the last launch_gemm call of this thread.
thread_local int t_gemm_launches = 0;

// Dynamic shared memory a kernel may request: the device's opt-in limit per
// block minus the kernel's static shared memory.
template <class K>
int query_dyn_smem_limit(K kern) {
    int dev = 0, optin = 0;
    cudaFuncAttributes fa{};
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        cudaFuncGetAttributes(&fa, kern) != cudaSuccess)
        return -1;
    return optin - static_cast<int>(fa.sharedSizeBytes);
}

// col0: output columns before this launch's first (column groups of a wide
// GEMM, below); p.out / p.res / p.res_scale already point at column col0.
template <int PRO, int EPI, int AMODE, int NT>
int launch_one(const GemmParams& p, cudaStream_t s, int col0 = 0) {
    auto kern = gemm_ws_kernel<PRO, EPI, AMODE, NT>;
    constexpr int kOutCols = (EPI == kEpiGate) ? NT / 2 : NT;
    using Stg = Staging<kOutCols>;
    using Plan = SmemPlan<PRO, EPI, NT, AMODE>;
    const int smem = Plan::bytes(p);
    static int limit = -1;  // per instantiation: its static shared memory differs
    if (limit < 0) limit = query_dyn_smem_limit(kern);
    if (limit < 0) return dn_fail(DN_ERR_CUDA, "gemm: kernel attributes");
    if (smem > limit) {
        // A wide N: the per-column parameter vectors (bias, LN fold, residual
        // scale) no longer fit beside the ring and the staging tile. Run
        // column groups of N tiles as separate launches, each with its slice
        // of B, of the vectors and of the output columns.
        constexpr bool kSplit = (AMODE == kARows || AMODE == kARowsPair) &&
                                (EPI == kEpiStore || EPI == kEpiGate || EPI == kEpiResidual);
        GemmParams q = p;
        int per = p.n_tiles;
        while (per > 1 && Plan::bytes(q) > limit) {
            per = (per + 1) / 2;
            q.n_tiles = per;
            q.n_out = std::min(p.n_out, per * kOutCols);
        }
        if (!kSplit || col0 != 0 || Plan::bytes(q) > limit)
            return dn_fail(DN_ERR_UNSUPPORTED, "gemm: tile does not fit in shared memory");
        int launched = 0;
        for (int t0 = 0; t0 < p.n_tiles; t0 += per) {
            const int c0 = t0 * kOutCols;
            if (c0 >= p.n_out) break;
            q = p;
            q.n_tiles = std::min(per, p.n_tiles - t0);
            q.bpack = p.bpack + static_cast<size_t>(t0) * p.k_chunks * gemm_btile_bytes(NT, p.KC);
            if (p.bias) q.bias = p.bias + static_cast<size_t>(t0) * NT;
            if (p.ln_c1) q.ln_c1 = p.ln_c1 + static_cast<size_t>(t0) * NT;
            q.out = p.out + c0;
            if (p.res) q.res = p.res + c0;
            if (p.res_scale) q.res_scale = p.res_scale + c0;
            q.n_out = std::min(p.n_out - c0, q.n_tiles * kOutCols);
            const int rc = launch_one<PRO, EPI, AMODE, NT>(q, s, c0);
            if (rc != DN_OK) return rc;
            ++launched;
        }
        t_gemm_launches = launched;
        return DN_OK;
    }
    t_gemm_launches = 1;
    static int configured = 0;  // largest dynamic footprint granted so far
    if (smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return dn_cuda_fail(e, "gemm: set smem attribute");
        configured = smem;
    }
    if (PRO == kProLayerNorm && !p.ln_c1) return dn_fail(DN_ERR_INVALID_ARG, "gemm: LN fold needs c1");
    GemmMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    constexpr bool kRowT = (AMODE == kAPairs) || (EPI == kEpiShuffleRows);
    if (kRowT && (p.Wo <= 0 || p.M % p.Wo != 0)) return dn_fail(DN_ERR_INVALID_ARG, "gemm: rows must be whole output rows");
    if (AMODE == kAPairs) {
        // Input [N * 2Ho rows][Wo pixel pairs][2 seg_c]: chunk j of K is row
        // 2y + ky, pair channels k0 .. k0 + KC.
        if (p.nseg != 1 || p.a_swz != p.KC * 2 || (2 * p.seg_c) % p.KC != 0 || p.K != 4 * p.seg_c)
            return dn_fail(DN_ERR_UNSUPPORTED, "gemm: pair loads need one source, a swizzled A and KC | 2C");
        const int rc = make_map3(&maps.a[0], p.a[0], static_cast<long long>(p.M / p.Wo) * 2, p.Wo, 2 * p.seg_c, p.KC,
                                 kRows, swizzle_for(p.a_swz));
        if (rc != DN_OK) return rc;
    } else if (AMODE != kAS2x2) {
        if (p.nseg > 1 && p.M != p.hw) return dn_fail(DN_ERR_UNSUPPORTED, "gemm: concat sources need one image");
        if (p.nseg == 1 && p.M != p.hw && p.a_img_stride != static_cast<long long>(p.hw) * p.seg_c)
            return dn_fail(DN_ERR_UNSUPPORTED, "gemm: batched A rows must be contiguous");
        if (p.a_swz && p.a_swz != p.KC * 2) return dn_fail(DN_ERR_INVALID_ARG, "gemm: A swizzle span must be KC*2");
        if (p.a_swz && p.nseg > 1 && p.seg_c < p.KC)
            return dn_fail(DN_ERR_INVALID_ARG, "gemm: swizzled concat needs KC <= segment width");
        for (int sgi = 0; sgi < p.nseg; ++sgi) {
            const int rc = p.a_swz ? make_map(&maps.a[sgi], p.a[sgi], p.M, p.seg_c, p.seg_c, p.KC, swizzle_for(p.a_swz))
                                   : make_map(&maps.a[sgi], p.a[sgi], p.M, p.seg_c, p.seg_c, 8, CU_TENSOR_MAP_SWIZZLE_NONE);
            if (rc != DN_OK) return rc;
        }
    }
    if (EPI == kEpiShuffleRows) {
        // Fine output and skip: [N * 2Ho rows][2 Wo][out_c], boxes of one
        // 256-pixel fine-row run of the tile.
        if (p.out_c * 4 != NT || (p.out_c != 32 && p.out_c != 64) || p.n_tiles != 1)
            return dn_fail(DN_ERR_UNSUPPORTED, "gemm: the staged shuffle needs NT = 4 * out_c, out_c 32 or 64");
        const long long frows = static_cast<long long>(p.M / p.Wo) * 2;
        int rc = make_map3(&maps.out, p.out, frows, 2 * p.Wo, p.out_c, p.out_c, 256, swizzle_for(p.out_c * 2));
        if (rc == DN_OK) rc = make_map3(&maps.res, p.skip, frows, 2 * p.Wo, p.out_c, p.out_c, 256, swizzle_for(p.out_c * 2));
        if (rc != DN_OK) return rc;
    } else if (EPI != kEpiShuffleAdd && p.out_c % kOutCols == 0) {
        int rc = kRowT ? make_map3(&maps.out, p.out, p.M / p.Wo, p.Wo, p.out_c, Stg::EB, kRows, swizzle_for(Stg::kRowBytes))
                       : make_map(&maps.out, p.out, p.M, p.out_c - col0, p.out_c, Stg::EB, swizzle_for(Stg::kRowBytes));
        if (rc != DN_OK) return rc;
        if (EPI == kEpiResidual) {
            rc = make_map(&maps.res, p.res, p.M, p.out_c - col0, p.out_c, Stg::EB, swizzle_for(Stg::kRowBytes));
            if (rc != DN_OK) return rc;
        }
    }
    constexpr bool kPair = (AMODE == kARowsPair);
    constexpr int kTileRows = kPair ? 2 * kRows : kRows;
    const int m_tiles = kRowT ? (p.M / p.Wo) * ((p.Wo + kRows - 1) / kRows) : (p.M + kTileRows - 1) / kTileRows;
    const long long tiles = static_cast<long long>(m_tiles) * p.n_tiles;
    // TMEM: 2 accumulators of NT columns each; at most 512 columns per SM.
    const int by_tmem = 512 / (2 * (NT < 32 ? 32 : NT));
    const int by_smem = (227 * 1024) / (smem + 2048);
    const int per_sm = std::max(1, std::min(by_tmem, by_smem));
    const dim3 block(PRO == kProLayerNorm ? kThreadsLN : kThreads);
    cudaError_t e;
    if (kPair) {
        // One cluster of two CTAs per pair tile, at most one pair per two SMs.
        const long long pairs = std::min<long long>(tiles, static_cast<long long>(num_sms() / 2) * per_sm);
        e = launch_pdl_pair(kern, dim3(static_cast<unsigned>(2 * pairs)), block, smem, s, p, maps);
    } else {
        const long long grid = std::min<long long>(tiles, static_cast<long long>(num_sms()) * per_sm);
        e = launch_pdl(kern, dim3(static_cast<unsigned>(grid)), block, smem, s, p, maps);
    }
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

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

int gemm_last_launches() { return t_gemm_launches; }

int launch_gemm(const GemmParams& p, int pro, int epi, int amode, int nt, cudaStream_t s) {
    t_gemm_launches = 0;
    if (p.KC != 16 && p.KC != 32 && p.KC != 64) return dn_fail(DN_ERR_UNSUPPORTED, "gemm: KC must be 16/32/64");
    if (p.a_swz != 0 && p.a_swz != 32 && p.a_swz != 64 && p.a_swz != 128)
        return dn_fail(DN_ERR_UNSUPPORTED, "gemm: bad A swizzle span");
    if (p.seg_c % 8 != 0) return dn_fail(DN_ERR_UNSUPPORTED, "gemm: channels must be a multiple of 8");
    if (p.M <= 0) return DN_OK;
    if (pro == kProLayerNorm && p.nseg != 1) return dn_fail(DN_ERR_UNSUPPORTED, "gemm: LN needs one source");
    if (p.nseg < 1 || p.nseg > kMaxSeg) return dn_fail(DN_ERR_INVALID_ARG, "gemm: bad segment count");
    // Instantiated combinations (the ones the planner emits).
    if (amode == kARowsPair) {  // CTA pairs: 128/256-wide tiles of the 1x1 convs
        if (p.nseg == 1 && (nt == 128 || nt == 256)) {
            const bool w = nt == 256;
            if (pro == kProLayerNorm && epi == kEpiStore)
                return w ? launch_one<kProLayerNorm, kEpiStore, kARowsPair, 256>(p, s)
                         : launch_one<kProLayerNorm, kEpiStore, kARowsPair, 128>(p, s);
            if (pro == kProLayerNorm && epi == kEpiGate)
                return w ? launch_one<kProLayerNorm, kEpiGate, kARowsPair, 256>(p, s)
                         : launch_one<kProLayerNorm, kEpiGate, kARowsPair, 128>(p, s);
            if (pro == kProScale && epi == kEpiResidual)
                return w ? launch_one<kProScale, kEpiResidual, kARowsPair, 256>(p, s)
                         : launch_one<kProScale, kEpiResidual, kARowsPair, 128>(p, s);
            if (pro == kProNone && epi == kEpiResidual)
                return w ? launch_one<kProNone, kEpiResidual, kARowsPair, 256>(p, s)
                         : launch_one<kProNone, kEpiResidual, kARowsPair, 128>(p, s);
            if (pro == kProNone && epi == kEpiStore)
                return w ? launch_one<kProNone, kEpiStore, kARowsPair, 256>(p, s)
                         : launch_one<kProNone, kEpiStore, kARowsPair, 128>(p, s);
        }
        amode = kARows;
    }
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
    if (amode == kAPairs && pro == kProNone && epi == kEpiStore)
        return launch_nt<kProNone, kEpiStore, kAPairs>(p, nt, s);
    if (amode == kARows && pro == kProNone && epi == kEpiShuffleRows) {
        if (nt == 128) return launch_one<kProNone, kEpiShuffleRows, kARows, 128>(p, s);
        if (nt == 256) return launch_one<kProNone, kEpiShuffleRows, kARows, 256>(p, s);
        return dn_fail(DN_ERR_UNSUPPORTED, "gemm: the staged shuffle needs a 128- or 256-wide tile");
    }
    return dn_fail(DN_ERR_UNSUPPORTED, "gemm: unsupported prologue/epilogue combination");
}

}  // namespace dnb
