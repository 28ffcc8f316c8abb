// Second pass of a deep NAFBlock (C = D = F = 128 or 256 channels) in one
// kernel:
//
//   y   = x + beta * (g (W3 diag(s))^T + b3)          conv3, SCA scale in W3
//   h   = SimpleGate(LN2(y) W4^T + b4)                 LN2 folded into W4
//   out = y + gamma * (h W5^T + b5)                    conv5
//
// the tail of the reference block (src/models/nafnet.cu:176-215:
// scaled add, LayerNorm, conv4, bias, gate, conv5, bias, scaled add;
// training/models.py:178-185), which the separate-GEMM path runs as three
// launches with y and h round-tripping through memory.
//
// Operands stream through a ring of 32 KB units, one mbarrier per unit: the
// cost of a unit is dominated by a per-copy latency that hardly depends on
// its size, so a few large units move far more bytes per microsecond than
// many small ones. Per 128-pixel tile:
//   C = 256: g goes straight into the y buffer (sY, the A of conv3); units:
//            conv3 K chunks (the whole [256 x 64] weight slice each), x (two
//            64-channel boxes per unit), conv4 per gate chunk (two K chunks
//            of the [a | b] slice), conv5 per gate chunk ([256 x 64]).
//   C = 128: units: conv3 K chunk [g box | weight slice], x, conv4 per gate
//            chunk, conv5 (both gate chunks in one unit).
// One CTA (416 threads) owns a stream of tiles:
//   warps 0, 10-12  producers: ring slot s is always filled by producer
//            s % 4 (a single issuing thread keeps only about one copy in
//            flight; one owner per slot keeps its empty-barrier waits in use
//            order, since a parity wait cannot tell a use two phases back);
//            producer 0 also loads g into sY (C = 256) once the previous
//            tile's output has left it.
//   warp 1   MMA issuer: conv3 into TMEM columns [0, C) (N = C); conv4 per
//            64-channel gate chunk j (a and b halves side by side, N = 128)
//            into one of two TMEM buffers at [C, C + 256); conv5 (N = C),
//            with the gated chunk as A, accumulating into its own columns
//            [C + 256, 2C + 256) when they fit (C = 128: the next tile's
//            conv3 then overlaps this tile's last epilogue), else into
//            conv3's (free by then). Issue order conv4_0, conv4_1, conv5_0,
//            conv4_2, conv5_1, ... so the next conv4 overlaps the epilogue of
//            the current chunk.
//   warps 2-9 epilogue, two threads per tile row (a TMEM lane) splitting its
//            columns: (1) y -> sY (fp16, the swizzled A of conv4) and the
//            LN2 statistics of the fp16 y (pairs merged with Chan's formula);
//            (2) per chunk h = (rstd*acc_a + c2a - rstd*mean*c1a) *
//            (rstd*acc_b + ...) -> sH[j % 2]; (3) out = y + gamma*(acc + b5)
//            written over y in sY, then TMA-stored.
// Per pixel this reads g and x and writes out (the 3C*2-byte minimum for the
// pass); weights stream from L2 once per tile. Every wait is bounded.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "fused_block.h"
#include "launch.cuh"
#include "sm100.cuh"
#include "status.h"

namespace dnb {

namespace {

constexpr int kDThreads = 416;  // warps 0, 10-12 producers, warp 1 MMA, warps 2-9 epilogue
constexpr int kProd = 4;        // producer warps
constexpr int kUnit = 32768;    // ring unit
constexpr int kBox = 16384;     // one [128 x 64] fp16 operand box

template <int C>
struct GeoD {
    static constexpr bool kGInY = C >= 256;          // g lands in sY (else it rides with conv3's weights)
    static constexpr int R = C >= 256 ? 3 : 4;       // ring units
    static constexpr int KC = C / 64;                // K chunks of conv3 and conv4 (K = C)
    static constexpr int J = C / 64;                 // 64-channel gate chunks (F = C)
    static constexpr int U3 = KC;                    // conv3 units
    static constexpr int UX = C / 128;               // x units (two boxes each)
    static constexpr int U4 = KC / 2;                // units per gate chunk (two K chunks each)
    static constexpr int U5 = C >= 256 ? J : 1;      // conv5 units (one per chunk, or both chunks)
    static constexpr int U = U3 + UX + J * U4 + U5;  // units per tile
    static constexpr int Y_BYTES = 128 * C * 2;
    static constexpr int H_BYTES = kBox;
    static constexpr int P_FLOATS = 4 * C + 4 * C;   // b3, beta, gamma, b5, c1[2F], c2[2F]
    static constexpr int SMEM = 1024 + Y_BYTES + 2 * H_BYTES + R * kUnit + P_FLOATS * 4;
    static constexpr int TMEM_COLS = 512;
    static constexpr bool kSplit = 2 * C + 256 <= 512;  // conv5 has columns of its own
    static constexpr int ACC5 = kSplit ? C + 256 : 0;   // conv5 accumulator column
    static_assert(C == 128 || C == 256, "tile geometry");
    static_assert(SMEM <= 227 * 1024, "shared memory");
    static_assert(U5 == J || J == 2, "conv5 chunks share a unit only as one pair");
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return p + ((1024u - (smem_u32(p) & 1023u)) & 1023u);
}

__device__ __forceinline__ void epi_sync() { named_sync(1, 256); }
__device__ __forceinline__ bool epi_sync_or(bool v) { return named_sync_or(1, 256, v); }

template <int C>
__global__ void __launch_bounds__(kDThreads, 1)
    deep_b_kernel(const __grid_constant__ DeepBParams p, const __grid_constant__ CUtensorMap mg,
                  const __grid_constant__ CUtensorMap mx, const __grid_constant__ CUtensorMap mo) {
    using G = GeoD<C>;
    if (threadIdx.x == 0) {
        prefetch_tmap(&mg);
        prefetch_tmap(&mx);
        prefetch_tmap(&mo);
    }
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    uint8_t* sY = smem;                   // C/64 boxes [128 x 64], 128-byte swizzle: (g,) y, out
    uint8_t* sH = sY + G::Y_BYTES;        // 2 gate chunks [128 x 64], same layout
    uint8_t* ring = sH + 2 * G::H_BYTES;  // R units
    float* sB3 = reinterpret_cast<float*>(ring + G::R * kUnit);
    float* sBeta = sB3 + C;
    float* sGam = sBeta + C;
    float* sB5 = sGam + C;
    float* sC1 = sB5 + C;  // [2F], packed order j*128 + (a: c, b: 64 + c)
    float* sC2 = sC1 + 2 * C;
    __shared__ uint64_t full[G::R], empty[G::R];
    __shared__ uint64_t acc3_full, y_ready, acc5_full, acc_free, mma_done, g_full, sy_free;
    __shared__ uint64_t acc4_full[2], acc4_empty[2], h_full[2], h_empty[2];
    __shared__ float2 s_stat[2][128];
    __shared__ uint32_t tslot;
    __shared__ volatile int s_abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tiles = (p.M + 127) / 128;

    for (int i = tid; i < C; i += kDThreads) {
        sB3[i] = p.b3[i];
        sBeta[i] = p.beta[i];
        sGam[i] = p.gamma[i];
        sB5[i] = p.b5[i];
    }
    for (int i = tid; i < 2 * C; i += kDThreads) {
        sC1[i] = p.c1[i];
        sC2[i] = p.c2[i];
    }
    if (warp == 0) {
        tmem_alloc(&tslot, G::TMEM_COLS);
        tmem_relinquish();
    }
    if (tid == 32) {
        for (int s = 0; s < G::R; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&acc3_full, 1);
        mbar_init(&y_ready, 1);
        mbar_init(&acc5_full, 1);
        mbar_init(&acc_free, 1);
        mbar_init(&mma_done, 1);
        mbar_init(&g_full, 1);
        mbar_init(&sy_free, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc4_full[b], 1);
            mbar_init(&acc4_empty[b], 1);
            mbar_init(&h_full[b], 1);
            mbar_init(&h_empty[b], 1);
        }
        s_abort = 0;
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    pdl_trigger();  // only once this CTA holds its TMEM columns
    pdl_wait();  // g, x and the SCA-scaled conv3 image come from earlier kernels

    if (warp == 0 || warp >= 10) {
        // ------------------------------ producers --------------------------------
        const int pk = warp == 0 ? 0 : warp - 9;
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            // Claims sequence unit `it`: the slot, once free, armed for a full
            // unit; nullptr if the slot belongs to another producer (or on
            // abort, with `ok` cleared).
            auto slot = [&](uint64_t*& bar) -> uint8_t* {
                const uint32_t v = it++;
                if (static_cast<int>((v % G::R) % kProd) != pk) return nullptr;
                const uint32_t s = v % G::R, ph = (v / G::R) & 1u;
                if (!wait_or_abort(&empty[s], ph ^ 1u, &s_abort, p.err, 0x50)) {
                    ok = false;
                    return nullptr;
                }
                bar = &full[s];
                mbar_arrive_expect_tx(bar, kUnit);
                return ring + s * kUnit;
            };
            int tl = 0;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tl) {
                const int m0 = t * 128;
                uint64_t* bar = nullptr;
                uint8_t* u;
                if (G::kGInY && pk == 0) {
                    // g of this tile into sY once the previous output has left it.
                    if (!wait_or_abort(&sy_free, (tl & 1) ^ 1, &s_abort, p.err, 0x51)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&g_full, G::Y_BYTES);
                    for (int kk = 0; kk < G::KC; ++kk) tma_load_2d(sY + kk * kBox, &mg, kk * 64, m0, &g_full);
                }
                for (int kk = 0; kk < G::U3 && ok; ++kk)
                    if ((u = slot(bar))) {
                        if (G::kGInY) {
                            bulk_g2s(u, p.w3 + static_cast<size_t>(kk) * kUnit, kUnit, bar);
                        } else {
                            tma_load_2d(u, &mg, kk * 64, m0, bar);
                            bulk_g2s(u + kBox, p.w3 + static_cast<size_t>(kk) * kBox, kBox, bar);
                        }
                    }
                for (int q = 0; q < G::UX && ok; ++q)
                    if ((u = slot(bar))) {
                        tma_load_2d(u, &mx, 128 * q, m0, bar);
                        tma_load_2d(u + kBox, &mx, 128 * q + 64, m0, bar);
                    }
                // conv4 chunk j: K chunks 2m, 2m+1 of its [a | b] slice (contiguous).
                auto c4 = [&](int j) {
                    for (int m = 0; m < G::U4 && ok; ++m)
                        if ((u = slot(bar)))
                            bulk_g2s(u, p.w4 + (static_cast<size_t>(j) * G::U4 + m) * kUnit, kUnit, bar);
                };
                // conv5: K chunk j of the [C x F] image (C = 256), or both chunks (C = 128).
                auto c5 = [&](int j) {
                    if ((u = slot(bar))) bulk_g2s(u, p.w5 + static_cast<size_t>(j) * kUnit, kUnit, bar);
                };
                c4(0);
                for (int j = 1; j < G::J && ok; ++j) {
                    c4(j);
                    if (G::U5 == G::J) c5(j - 1);
                    else if (j == 1) c5(0);
                }
                if (G::U5 == G::J && ok) c5(G::J - 1);
            }
            if (!ok) {
                // Let the copies already issued land before the CTA's memory is released.
                const uint32_t lo = it > static_cast<uint32_t>(G::R) ? it - G::R : 0u;
                for (uint32_t v = lo; v + 1 < it; ++v)
                    if (static_cast<int>((v % G::R) % kProd) == pk) mbar_wait(&full[v % G::R], (v / G::R) & 1u, 5000000ull);
            }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer -------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc128 = idesc_f16_f32(128, 128);
            constexpr uint32_t idescC = idesc_f16_f32(128, C);
            uint32_t it = 0, n4 = 0;
            bool ok = true;
            auto take = [&](uint32_t site) -> uint32_t {
                const uint32_t s = it % G::R, ph = (it / G::R) & 1u;
                ++it;
                if (ok && !wait_or_abort(&full[s], ph, &s_abort, p.err, site)) ok = false;
                return s;
            };
            // Descriptors are built once; each MMA adds byte offsets to them.
            const uint64_t d_ring_b = sdesc_kmajor(smem_u32(ring), 128, 1024);
            const uint64_t d_ring_a = sdesc_kmajor_sw(smem_u32(ring), 128);
            const uint64_t d_y = sdesc_kmajor_sw(smem_u32(sY), 128);
            const uint64_t d_h = sdesc_kmajor_sw(smem_u32(sH), 128);
            auto bdesc = [&](uint32_t s, uint32_t off, int k) {
                return desc_add(d_ring_b, s * kUnit + off + k * 256);
            };
            int tl = 0;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tl) {
                // conv3 overwrites [0, C): with a shared accumulator the
                // previous tile's output epilogue must have drained it.
                if (!G::kSplit && !wait_or_abort(&acc_free, (tl & 1) ^ 1, &s_abort, p.err, 0x52)) break;
                if (G::kGInY && !wait_or_abort(&g_full, tl & 1, &s_abort, p.err, 0x53)) break;
                tc_fence_after();
                // conv3: [128 x C] x [C -> C]
                for (int kk = 0; kk < G::U3 && ok; ++kk) {
                    const uint32_t s = take(0x54);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t a0 = G::kGInY ? desc_add(d_y, kk * kBox) : desc_add(d_ring_a, s * kUnit);
                    const uint32_t boff = G::kGInY ? 0u : static_cast<uint32_t>(kBox);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        mma_f16(tmem, desc_add(a0, k * 32), bdesc(s, boff, k), idescC, (kk | k) ? 1u : 0u);
                    mma_commit(&empty[s]);
                }
                if (!ok) break;
                mma_commit(&acc3_full);
                it += G::UX;  // the x units go to the epilogue
                if (!wait_or_abort(&y_ready, tl & 1, &s_abort, p.err, 0x55)) break;
                tc_fence_after();
                auto c4 = [&](int j) {
                    const uint32_t u4 = n4 + j, b = u4 & 1u;
                    if (!wait_or_abort(&acc4_empty[b], ((u4 >> 1) & 1u) ^ 1u, &s_abort, p.err, 0x56)) {
                        ok = false;
                        return;
                    }
                    tc_fence_after();
                    for (int m = 0; m < G::U4; ++m) {
                        const uint32_t s = take(0x57);
                        if (!ok) return;
                        tc_fence_after();
#pragma unroll
                        for (int kc = 0; kc < 2; ++kc) {
                            const int kk = 2 * m + kc;
                            const uint64_t a0 = desc_add(d_y, kk * kBox);
#pragma unroll
                            for (int k = 0; k < 4; ++k)
                                mma_f16(tmem + C + b * 128, desc_add(a0, k * 32), bdesc(s, kc * kBox, k), idesc128,
                                        (kk | k) ? 1u : 0u);
                        }
                        mma_commit(&empty[s]);
                    }
                    mma_commit(&acc4_full[b]);
                };
                uint32_t s5 = 0;  // C = 128: the unit holding both conv5 chunks
                auto c5 = [&](int j) {
                    const uint32_t u4 = n4 + j, b = u4 & 1u;
                    // Own conv5 columns: the previous tile's output epilogue
                    // must have drained them before the first chunk overwrites.
                    if (G::kSplit && j == 0 && !wait_or_abort(&acc_free, (tl & 1) ^ 1, &s_abort, p.err, 0x52)) {
                        ok = false;
                        return;
                    }
                    if (!wait_or_abort(&h_full[b], (u4 >> 1) & 1u, &s_abort, p.err, 0x58)) {
                        ok = false;
                        return;
                    }
                    uint32_t s, off;
                    if (G::U5 == G::J) {
                        s = take(0x59);
                        off = 0;
                    } else {
                        if (j == 0) s5 = take(0x59);
                        s = s5;
                        off = static_cast<uint32_t>(j) * kBox;
                    }
                    if (!ok) return;
                    tc_fence_after();
                    const uint64_t a0 = desc_add(d_h, b * G::H_BYTES);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        mma_f16(tmem + G::ACC5, desc_add(a0, k * 32), bdesc(s, off, k), idescC, (j | k) ? 1u : 0u);
                    if (G::U5 == G::J || j == G::J - 1) mma_commit(&empty[s]);
                    mma_commit(&h_empty[b]);
                };
                c4(0);
                for (int j = 1; j < G::J && ok; ++j) {
                    c4(j);
                    if (ok) c5(j - 1);
                }
                if (ok) c5(G::J - 1);
                if (!ok) break;
                mma_commit(&acc5_full);
                n4 += G::J;
            }
            // Every MMA of this CTA has completed before TMEM is released.
            mma_commit(&mma_done);
            mbar_wait(&mma_done, 0, 5000000ull);
        }
    } else {
        // ------------------------------ epilogue ---------------------------------
        const int q = warp & 3;            // TMEM lane quarter of this warp
        const int half = (warp - 2) >> 2;  // column half of the tile row
        const int r = q * 32 + lane;       // tile row == TMEM lane
        const bool leader = (tid == 64);
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
        constexpr int CH = C / 2;
        const int cb = half * CH;
        const float2 one2 = make_float2(1.f, 1.f);
        uint32_t it_base = 0, n4 = 0;
        int tl = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++tl, it_base += G::U) {
            const int m0 = t * 128;
            // (1) y = x + beta * (acc + b3) -> sY; LN2 statistics of the fp16 y.
            bool ok = wait_or_abort(&acc3_full, tl & 1, &s_abort, p.err, 0x5a);
            for (int kq = 0; kq < G::UX && ok; ++kq) {
                const uint32_t v = it_base + G::U3 + kq;
                ok = wait_or_abort(&full[v % G::R], (v / G::R) & 1u, &s_abort, p.err, 0x5b);
            }
            if (leader) bulk_wait_read0();  // the previous tile's output has left sY
            if (epi_sync_or(!ok)) break;
            tc_fence_after();
            float sh = 0.f, s1 = 0.f, s2 = 0.f;
#pragma unroll 1
            for (int c0 = cb; c0 < cb + CH; c0 += 16) {
                float v[16];
                tmem_ld16(lane_base + c0, v);
                tmem_ld_wait();
                const int box = c0 >> 6;
                const uint8_t* xu = ring + ((it_base + G::U3 + (box >> 1)) % G::R) * kUnit + (box & 1) * kBox;
                uint8_t* yb = sY + box * kBox;
#pragma unroll
                for (int g2 = 0; g2 < 2; ++g2) {
                    const uint32_t off = sw_offset(r, ((c0 & 63) >> 3) + g2, 128);
                    const uint4 xv = *reinterpret_cast<const uint4*>(xu + off);
                    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
                    const int c = c0 + 8 * g2;
                    const float4 bb0 = *reinterpret_cast<const float4*>(sB3 + c);
                    const float4 bb1 = *reinterpret_cast<const float4*>(sB3 + c + 4);
                    const float4 be0 = *reinterpret_cast<const float4*>(sBeta + c);
                    const float4 be1 = *reinterpret_cast<const float4*>(sBeta + c + 4);
                    const float2 bb[4] = {make_float2(bb0.x, bb0.y), make_float2(bb0.z, bb0.w),
                                          make_float2(bb1.x, bb1.y), make_float2(bb1.z, bb1.w)};
                    const float2 be[4] = {make_float2(be0.x, be0.y), make_float2(be0.z, be0.w),
                                          make_float2(be1.x, be1.y), make_float2(be1.z, be1.w)};
                    uint32_t o[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float2 a = ffma2(make_float2(v[8 * g2 + 2 * i], v[8 * g2 + 2 * i + 1]), one2, bb[i]);
                        const float2 y = ffma2(be[i], a, unpack_half2(xw[i]));
                        o[i] = pack_half2(y.x, y.y);
                        const float2 yr = unpack_half2(o[i]);  // statistics of the stored fp16 y
                        if (c0 == cb && g2 == 0 && i == 0) sh = yr.x;
                        const float d0 = yr.x - sh, d1 = yr.y - sh;
                        s1 += d0 + d1;
                        s2 = fmaf(d0, d0, fmaf(d1, d1, s2));
                    }
                    *reinterpret_cast<uint4*>(yb + off) = make_uint4(o[0], o[1], o[2], o[3]);
                }
            }
            const float m_h = sh + s1 * (1.0f / CH);
            const float M2 = fmaxf(s2 - s1 * s1 * (1.0f / CH), 0.f);
            s_stat[half][r] = make_float2(m_h, M2);
            fence_async_smem();  // y is conv4's A (async proxy)
            tc_fence_before();
            epi_sync();
            const float2 other = s_stat[half ^ 1][r];
            const float mean = 0.5f * (m_h + other.x);
            const float dm = m_h - other.x;
            const float var = (M2 + other.y + dm * dm * (0.25f * C)) * (1.0f / C);
            const float rstd = rsqrtf(var + 1e-6f);
            if (leader) {
                mbar_arrive(&y_ready);
                for (int kq = 0; kq < G::UX; ++kq) mbar_arrive(&empty[(it_base + G::U3 + kq) % G::R]);
            }
            // (2) gate chunks: h = (LN-folded a) * (LN-folded b) -> sH[j % 2].
            const float2 rs2 = make_float2(rstd, rstd), nm2 = make_float2(-rstd * mean, -rstd * mean);
            auto fold8 = [&](const float* acc, int n, float2 (&out)[4]) {
                const float4 k0 = *reinterpret_cast<const float4*>(sC1 + n);
                const float4 k1 = *reinterpret_cast<const float4*>(sC1 + n + 4);
                const float4 q0 = *reinterpret_cast<const float4*>(sC2 + n);
                const float4 q1 = *reinterpret_cast<const float4*>(sC2 + n + 4);
                const float2 kc[4] = {make_float2(k0.x, k0.y), make_float2(k0.z, k0.w), make_float2(k1.x, k1.y),
                                      make_float2(k1.z, k1.w)};
                const float2 qc[4] = {make_float2(q0.x, q0.y), make_float2(q0.z, q0.w), make_float2(q1.x, q1.y),
                                      make_float2(q1.z, q1.w)};
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    out[i] = ffma2(rs2, make_float2(acc[2 * i], acc[2 * i + 1]), ffma2(nm2, kc[i], qc[i]));
            };
            for (int j = 0; j < G::J && ok; ++j) {
                const uint32_t u4 = n4 + j, b = u4 & 1u;
                bool got = wait_or_abort(&acc4_full[b], (u4 >> 1) & 1u, &s_abort, p.err, 0x5c);
                if (got) got = wait_or_abort(&h_empty[b], ((u4 >> 1) & 1u) ^ 1u, &s_abort, p.err, 0x5d);
                if (epi_sync_or(!got)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int pa = j * 128;  // packed index of gate channel 64j (a); b at +64
                uint8_t* hb = sH + b * G::H_BYTES;
#pragma unroll
                for (int cc = half * 32; cc < half * 32 + 32; cc += 16) {
                    float va[16], vb[16];
                    tmem_ld16(lane_base + C + b * 128 + cc, va);
                    tmem_ld16(lane_base + C + b * 128 + 64 + cc, vb);
                    tmem_ld_wait();
#pragma unroll
                    for (int g2 = 0; g2 < 2; ++g2) {
                        float2 xa[4], xb[4];
                        fold8(va + 8 * g2, pa + cc + 8 * g2, xa);
                        fold8(vb + 8 * g2, pa + 64 + cc + 8 * g2, xb);
                        const float2 z = make_float2(0.f, 0.f);
                        uint32_t o[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float2 pr = ffma2(xa[i], xb[i], z);
                            o[i] = pack_half2(pr.x, pr.y);
                        }
                        *reinterpret_cast<uint4*>(hb + sw_offset(r, (cc >> 3) + g2, 128)) =
                            make_uint4(o[0], o[1], o[2], o[3]);
                    }
                }
                fence_async_smem();
                tc_fence_before();
                epi_sync();
                if (leader) {
                    mbar_arrive(&acc4_empty[b]);
                    mbar_arrive(&h_full[b]);
                }
            }
            if (!ok) break;
            n4 += G::J;
            // (3) out = y + gamma * (acc + b5), over y in sY, then TMA store.
            ok = wait_or_abort(&acc5_full, tl & 1, &s_abort, p.err, 0x5e);
            if (epi_sync_or(!ok)) break;
            tc_fence_after();
#pragma unroll 1
            for (int c0 = cb; c0 < cb + CH; c0 += 16) {
                float v[16];
                tmem_ld16(lane_base + G::ACC5 + c0, v);
                tmem_ld_wait();
                uint8_t* yb = sY + (c0 >> 6) * kBox;
#pragma unroll
                for (int g2 = 0; g2 < 2; ++g2) {
                    uint4* ptr = reinterpret_cast<uint4*>(yb + sw_offset(r, ((c0 & 63) >> 3) + g2, 128));
                    const uint4 yv = *ptr;
                    const uint32_t yw[4] = {yv.x, yv.y, yv.z, yv.w};
                    const int c = c0 + 8 * g2;
                    const float4 bb0 = *reinterpret_cast<const float4*>(sB5 + c);
                    const float4 bb1 = *reinterpret_cast<const float4*>(sB5 + c + 4);
                    const float4 ga0 = *reinterpret_cast<const float4*>(sGam + c);
                    const float4 ga1 = *reinterpret_cast<const float4*>(sGam + c + 4);
                    const float2 bb[4] = {make_float2(bb0.x, bb0.y), make_float2(bb0.z, bb0.w),
                                          make_float2(bb1.x, bb1.y), make_float2(bb1.z, bb1.w)};
                    const float2 ga[4] = {make_float2(ga0.x, ga0.y), make_float2(ga0.z, ga0.w),
                                          make_float2(ga1.x, ga1.y), make_float2(ga1.z, ga1.w)};
                    uint32_t o[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float2 a = ffma2(make_float2(v[8 * g2 + 2 * i], v[8 * g2 + 2 * i + 1]), one2, bb[i]);
                        const float2 y = ffma2(ga[i], a, unpack_half2(yw[i]));
                        o[i] = pack_half2(y.x, y.y);
                    }
                    *ptr = make_uint4(o[0], o[1], o[2], o[3]);
                }
            }
            fence_async_smem();
            tc_fence_before();
            epi_sync();
            if (leader) {
                mbar_arrive(&acc_free);
                for (int bx = 0; bx < C / 64; ++bx) tma_store_2d(&mo, bx * 64, m0, sY + bx * kBox);
                bulk_commit();
                if (G::kGInY) {
                    bulk_wait_read0();  // the output has left sY: the next tile's g may land there
                    mbar_arrive(&sy_free);
                }
            }
        }
        if (leader) bulk_wait0();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, G::TMEM_COLS);
}

template <int C>
int run_deep_b(const DeepBParams& p, cudaStream_t s) {
    using G = GeoD<C>;
    auto kern = deep_b_kernel<C>;
    static bool cfg = false;
    if (!cfg) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM);
        if (e != cudaSuccess) return dn_cuda_fail(e, "deep_b: smem attribute");
        cfg = true;
    }
    CUtensorMap mg, mx, mo;
    const cuuint32_t box[2] = {64, 128};
    const cuuint64_t dC[2] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(p.M)};
    const cuuint64_t sC[1] = {static_cast<cuuint64_t>(C) * 2};
    int rc = encode_f16_map(&mg, 2, p.g, dC, sC, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc == DN_OK) rc = encode_f16_map(&mx, 2, p.x, dC, sC, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc == DN_OK) rc = encode_f16_map(&mo, 2, p.out, dC, sC, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != DN_OK) return rc;
    const int tiles = (p.M + 127) / 128;
    const int grid = std::min(tiles, sm_count());
    cudaError_t e = launch_pdl(kern, dim3(grid), dim3(kDThreads), G::SMEM, s, p, mg, mx, mo);
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "deep_b: launch");
}

}  // namespace

bool deep_b_supported(int C, int D, int F) { return (C == 128 || C == 256) && D == C && F == C; }

int launch_deep_b(const DeepBParams& p, int C, int D, int F, cudaStream_t s) {
    if (p.M <= 0) return dn_fail(DN_ERR_INVALID_ARG, "deep_b: empty input");
    if (!deep_b_supported(C, D, F)) return dn_fail(DN_ERR_UNSUPPORTED, "deep_b: channel configuration");
    return C == 128 ? run_deep_b<128>(p, s) : run_deep_b<256>(p, s);
}

}  // namespace dnb
