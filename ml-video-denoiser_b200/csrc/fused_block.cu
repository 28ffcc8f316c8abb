// Fused NAFBlock for the HBM-bound shallow levels (C <= 64 channels), as the
// two passes the SCA global pool forces:
//
// Phase A (one CTA = a stream of TH x TW output tiles):
//   TMA loads the (TH+2) x (TW+2) halo of x (NHWC, zero outside the image)
//   straight into the swizzled K-major UMMA layout; one thread per halo pixel
//   normalises it in place (LayerNorm without the affine, FP32 statistics,
//   FP16 result as in the reference); tcgen05 runs conv1 over the halo
//   (M = 128 pixels per block, N = 2*dw, K = C) with the affine folded into
//   the weights (B = gamma*W1, bias' = b1 + W1 beta), and all eight warps
//   move u = acc + bias' (zero outside the image = the DW zero padding) to
//   shared memory; CUDA cores then run the 3x3 depthwise conv + bias +
//   SimpleGate (a thread owns 4 channels of one gate half and a 2 x 4 block
//   of outputs, so each loaded u vector feeds up to 6 outputs), write g by
//   TMA store and accumulate the per-image pool partials (deterministic).
// Phase B (one CTA = a stream of 128-pixel tiles): TMA brings g and x;
//   g *= s (SCA scale) in place; tcgen05 conv3 -> y = x + beta*(acc + b3)
//   (kept in registers) -> LayerNorm2 -> tcgen05 conv4 -> SimpleGate ->
//   tcgen05 conv5 -> out = y + gamma*(acc + b5) -> TMA store. All three
//   weight matrices stay resident in shared memory; the accumulators chain
//   through TMEM.
//
// Per pixel this moves x (plus halo) in, g out, g and x in, x' out: the
// two-pass minimum of 5C*2 bytes, against the ~14 passes of
// the reference block (src/models/nafnet.cu:146-215: LN, conv1, bias, conv2,
// bias, gate, pool, sca conv, scale, conv3, bias, scaled add, LN, conv4,
// bias, gate, conv5, bias, scaled add).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <string>

#include "fused_block.h"
#include "launch.cuh"
#include "sm100.cuh"
#include "status.h"

namespace dnb {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();  // gemm_tc.cu

namespace {

constexpr int kAThreads = 256;

constexpr int pow2_at_least(int v) {
    int p = 32;
    while (p < v) p <<= 1;
    return p;
}

template <int C, int D>
struct GeoA {
    static constexpr int TH = C <= 32 ? 8 : 4;
    static constexpr int TW = C <= 32 ? 32 : 16;
    static constexpr int HH = TH + 2;
    static constexpr int WW = TW + 2;
    static constexpr int P = HH * WW;                 // halo pixels
    static constexpr int NB = (P + 127) / 128;        // 128-row MMA blocks over the halo
    static constexpr int N1 = 2 * D;                  // conv1 outputs
    static constexpr int TMEM_COLS = pow2_at_least(NB * N1);
    static constexpr int ROWB = C * 2;                // A row bytes = TMA swizzle span
    static constexpr int A_BYTES = NB * 128 * ROWB;
    static constexpr int U_PITCH = N1 * 2 + 16;       // padded: conflict-free DW reads
    static constexpr int U_BYTES = ((P * U_PITCH + 1023) / 1024) * 1024;
    static constexpr int G_BYTES = TH * TW * D * 2;
    static constexpr int W1_BYTES = N1 * C * 2;       // one K chunk (C <= 64)
    // depthwise: thread = (gate half, 4-channel group, slot); slot = 2 x 4 output block
    static constexpr int CG = D / 4;
    static constexpr int SLOTS = kAThreads / (2 * CG);
    static constexpr int NBLK = (TH / 2) * (TW / 4);
    // floats: bias' [2D], pool partials [8][D], pool reduction [2*SLOTS][D]
    static constexpr int F_FLOATS = N1 + 8 * D + 2 * SLOTS * D;
    static constexpr int SMEM = 1024 + A_BYTES + U_BYTES + G_BYTES + W1_BYTES + F_FLOATS * 4;
    static_assert(TH % 2 == 0 && TW % 4 == 0, "2 x 4 output blocks");
};

template <int C, int D, int F>
struct GeoB {
    // conv3, conv4 and conv5 take turns on the same columns (each accumulator
    // is drained before the next MMA is issued), so more CTAs share an SM.
    static constexpr int TMEM_COLS = pow2_at_least(C > 2 * F ? C : 2 * F);
    static constexpr int G_BYTES = 128 * D * 2;
    static constexpr int X_BYTES = 128 * C * 2;
    static constexpr int A3_BYTES = 128 * F * 2;
    static constexpr int W3_BYTES = C * D * 2;
    static constexpr int W4_BYTES = 2 * F * C * 2;
    static constexpr int W5_BYTES = C * F * 2;
    static constexpr int F_FLOATS = 6 * C + 2 * F + 8 * D;
    // x, LN2(y) (which doubles as the output staging tile once conv4 has read it)
    static constexpr int SMEM = 1024 + G_BYTES + 2 * X_BYTES + A3_BYTES + W3_BYTES + W4_BYTES + W5_BYTES +
                                F_FLOATS * 4;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return p + ((1024u - (smem_u32(p) & 1023u)) & 1023u);
}

// Bounded wait; on expiry records `site` and returns false.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t site) {
    if (mbar_wait(bar, parity)) return true;
    report_error(err, site, kErrMbarTimeout);
    return false;
}

// ============================== phase A =====================================

template <int C, int D>
__global__ void __launch_bounds__(kAThreads, 2)
    fused_a_kernel(const __grid_constant__ FusedAParams p, const __grid_constant__ CUtensorMap mx,
                   const __grid_constant__ CUtensorMap mg) {
    using G = GeoA<C, D>;
    if (threadIdx.x == 0) {
        prefetch_tmap(&mx);
        prefetch_tmap(&mg);
    }
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    uint8_t* sA = smem;
    uint8_t* sU = sA + G::A_BYTES;
    uint8_t* sGo = sU + G::U_BYTES;
    uint8_t* sW1 = sGo + G::G_BYTES;
    float* sC2 = reinterpret_cast<float*>(sW1 + G::W1_BYTES);  // [2D]
    float* sPart = sC2 + G::N1;                                 // [8][D]
    float* sRed = sPart + 8 * D;                                // [2*SLOTS][D]
    __shared__ uint64_t bar_x, bar_w, bar_mma;
    __shared__ uint32_t tslot;
    __shared__ int s_fail;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tiles_x = (p.W + G::TW - 1) / G::TW;
    const int tiles_y = (p.H + G::TH - 1) / G::TH;
    const int per_img = tiles_x * tiles_y;
    const int total = per_img * p.N;
    auto decode = [&](int t, int& img, int& ty0, int& tx0) {
        img = t / per_img;
        const int r = t - img * per_img;
        ty0 = (r / tiles_x) * G::TH;
        tx0 = (r % tiles_x) * G::TW;
    };

    for (int i = tid; i < G::N1; i += kAThreads) sC2[i] = p.c2[i];
    for (int i = tid; i < 8 * D; i += kAThreads) sPart[i] = 0.f;
    if (warp == 0) {
        tmem_alloc(&tslot, G::TMEM_COLS);
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(&bar_x, 1);
        mbar_init(&bar_w, 1);
        mbar_init(&bar_mma, 1);
        s_fail = 0;
        fence_mbar_init();
        mbar_arrive_expect_tx(&bar_w, G::W1_BYTES);
        bulk_g2s(sW1, p.w1, G::W1_BYTES, &bar_w);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    pdl_trigger();  // only once this CTA holds its TMEM columns
    const uint64_t da1 = sdesc_kmajor_sw(smem_u32(sA), G::ROWB);
    const uint64_t db1 = sdesc_kmajor(smem_u32(sW1), 128, (C / 8) * 128);
    pdl_wait();  // x was written by the previous kernel
    if (tid == 0 && blockIdx.x < total) {
        int img, ty0, tx0;
        decode(blockIdx.x, img, ty0, tx0);
        mbar_arrive_expect_tx(&bar_x, G::P * G::ROWB);
        tma_load_4d(sA, &mx, 0, tx0 - 1, ty0 - 1, img, &bar_x);
    }
    const bool ok = __syncthreads_and(wait_bar(&bar_w, 0, p.err, 0x30)) != 0;

    // Depthwise mapping: gate half fastest (pairs meet through one shuffle),
    // then 4-channel group, then block slot.
    const int half = tid & 1;
    const int cg = (tid >> 1) % G::CG;
    const int slot = (tid >> 1) / G::CG;
    const int cin = half * D + cg * 4;
    float2 dww[9][2];
    float2 dwb[2];
#pragma unroll
    for (int tp = 0; tp < 9; ++tp)
#pragma unroll
        for (int i = 0; i < 2; ++i)
            dww[tp][i] = make_float2(p.dw_w[tp * G::N1 + cin + 2 * i], p.dw_w[tp * G::N1 + cin + 2 * i + 1]);
#pragma unroll
    for (int i = 0; i < 2; ++i) dwb[i] = make_float2(p.dw_b[cin + 2 * i], p.dw_b[cin + 2 * i + 1]);
    float ps[4] = {0.f, 0.f, 0.f, 0.f};

    int it = 0;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
        int img, ty0, tx0;
        decode(t, img, ty0, tx0);
        if (!wait_bar(&bar_x, it & 1, p.err, 0x31)) s_fail = 1;
        __syncthreads();
        if (s_fail) break;
        // (1) LayerNorm (no affine) of every halo pixel, in place: the row is
        // read once into registers; statistics are shifted sums (shift = its
        // first element) in two packed chains.
        for (int r = tid; r < G::P; r += kAThreads) {
            uint4 v[C / 8];
#pragma unroll
            for (int q = 0; q < C / 8; ++q) v[q] = *reinterpret_cast<const uint4*>(sA + sw_offset(r, q, G::ROWB));
            const float x0 = unpack_half2(v[0].x).x;
            const float2 nx = make_float2(-x0, -x0), one = make_float2(1.f, 1.f);
            float2 a1[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
            float2 a2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
            for (int q = 0; q < C / 8; ++q) {
                const uint32_t w[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 d = ffma2(unpack_half2(w[i]), one, nx);
                    a1[i & 1] = ffma2(d, one, a1[i & 1]);
                    a2[i & 1] = ffma2(d, d, a2[i & 1]);
                }
            }
            const float dm = ((a1[0].x + a1[0].y) + (a1[1].x + a1[1].y)) * (1.0f / C);
            const float var = fmaxf(((a2[0].x + a2[0].y) + (a2[1].x + a2[1].y)) * (1.0f / C) - dm * dm, 0.f);
            const float rstd = rsqrtf(var + 1e-6f);
            const float2 rs2 = make_float2(rstd, rstd);
            const float2 sh2 = make_float2(-(x0 + dm) * rstd, -(x0 + dm) * rstd);
#pragma unroll
            for (int q = 0; q < C / 8; ++q) {
                const uint32_t w[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
                uint32_t o[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 y = ffma2(unpack_half2(w[i]), rs2, sh2);
                    o[i] = pack_half2(y.x, y.y);
                }
                *reinterpret_cast<uint4*>(sA + sw_offset(r, q, G::ROWB)) = make_uint4(o[0], o[1], o[2], o[3]);
            }
        }
        fence_async_smem();  // the normalised rows feed the tensor core (async proxy)
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            constexpr uint32_t idesc = idesc_f16_f32(128, G::N1);
#pragma unroll
            for (int b = 0; b < G::NB; ++b)
#pragma unroll
                for (int k = 0; k < C / 16; ++k)
                    mma_f16(tmem + b * G::N1, desc_add(da1, b * 128 * G::ROWB + k * 32), desc_add(db1, k * 256), idesc,
                            k > 0 ? 1u : 0u);
            mma_commit(&bar_mma);
        }
        if (!wait_bar(&bar_mma, it & 1, p.err, 0x32)) s_fail = 1;
        tc_fence_after();
        // The halo tile is consumed: prefetch the next one.
        if (tid == 0 && !s_fail && t + static_cast<int>(gridDim.x) < total) {
            int ni, ny, nx2;
            decode(t + gridDim.x, ni, ny, nx2);
            mbar_arrive_expect_tx(&bar_x, G::P * G::ROWB);
            tma_load_4d(sA, &mx, 0, nx2 - 1, ny - 1, ni, &bar_x);
        }
        // (2) conv1 epilogue over all eight warps: warp w reads TMEM lane
        // quarter w%4 and every other 16-column chunk: u = acc + bias',
        // zero outside the image.
        {
            constexpr int CH = G::N1 / 16;
            const int q4 = warp & 3;
            for (int j = warp >> 2; j < G::NB * CH; j += 2) {
                const int b = j / CH, c0 = (j - b * CH) * 16;
                const int r = b * 128 + q4 * 32 + lane;
                float v[16];
                tmem_ld16(tmem + b * G::N1 + c0 + (static_cast<uint32_t>(q4 * 32) << 16), v);
                tmem_ld_wait();
                if (r >= G::P) continue;
                const int yy = ty0 - 1 + r / G::WW;
                const int xx = tx0 - 1 + r % G::WW;
                const bool inside = yy >= 0 && yy < p.H && xx >= 0 && xx < p.W;
                uint32_t pk[8];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float4 c = *reinterpret_cast<const float4*>(sC2 + c0 + 4 * i);
                    pk[2 * i] = inside ? pack_half2(v[4 * i] + c.x, v[4 * i + 1] + c.y) : 0u;
                    pk[2 * i + 1] = inside ? pack_half2(v[4 * i + 2] + c.z, v[4 * i + 3] + c.w) : 0u;
                }
                uint4* dst = reinterpret_cast<uint4*>(sU + r * G::U_PITCH + c0 * 2);
                dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
            }
        }
        tc_fence_before();
        if (tid == 0) bulk_wait_read0();  // the previous g tile has left sGo
        __syncthreads();
        // (3) Depthwise 3x3 + bias + SimpleGate. Block = output rows by, by+1 x
        // columns bx .. bx+3: halo rows by .. by+3 x columns bx .. bx+5 stream
        // through once; each loaded vector feeds every output it touches.
        for (int blk = slot; blk < G::NBLK; blk += G::SLOTS) {
            const int by = (blk / (G::TW / 4)) * 2, bx = (blk % (G::TW / 4)) * 4;
            float2 acc[2][4][2];
#pragma unroll
            for (int ro = 0; ro < 2; ++ro)
#pragma unroll
                for (int oc = 0; oc < 4; ++oc) {
                    acc[ro][oc][0] = dwb[0];
                    acc[ro][oc][1] = dwb[1];
                }
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) {
                float2 in[6][2];
                const uint8_t* row = sU + ((by + rr) * G::WW + bx) * G::U_PITCH + cin * 2;
#pragma unroll
                for (int cc = 0; cc < 6; ++cc) {
                    const uint2 u2 = *reinterpret_cast<const uint2*>(row + cc * G::U_PITCH);
                    in[cc][0] = unpack_half2(u2.x);
                    in[cc][1] = unpack_half2(u2.y);
                }
#pragma unroll
                for (int oc = 0; oc < 4; ++oc)
#pragma unroll
                    for (int kx = 0; kx < 3; ++kx)
#pragma unroll
                        for (int i = 0; i < 2; ++i) {
                            if (rr <= 2) acc[0][oc][i] = ffma2(in[oc + kx][i], dww[rr * 3 + kx][i], acc[0][oc][i]);
                            if (rr >= 1)
                                acc[1][oc][i] = ffma2(in[oc + kx][i], dww[(rr - 1) * 3 + kx][i], acc[1][oc][i]);
                        }
            }
            // Gate: this lane stores columns 2*half, 2*half+1 of both rows;
            // it hands the partner the other two columns' values.
#pragma unroll
            for (int ro = 0; ro < 2; ++ro)
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    const int oy = by + ro, ox = bx + 2 * half + k;
                    float2 prod[2];
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        const float2 lo = acc[ro][k][i], hi = acc[ro][2 + k][i];
                        const float2 mine = half ? hi : lo;
                        const float2 give = half ? lo : hi;
                        const float gx = __shfl_xor_sync(0xffffffffu, give.x, 1);
                        const float gy = __shfl_xor_sync(0xffffffffu, give.y, 1);
                        prod[i] = make_float2(mine.x * gx, mine.y * gy);
                    }
                    const uint32_t h01 = pack_half2(prod[0].x, prod[0].y), h23 = pack_half2(prod[1].x, prod[1].y);
                    *reinterpret_cast<uint2*>(sGo + ((oy * G::TW + ox) * D + cg * 4) * 2) = make_uint2(h01, h23);
                    if (ty0 + oy < p.H && tx0 + ox < p.W) {  // pool the stored fp16 values
                        const float2 f01 = unpack_half2(h01), f23 = unpack_half2(h23);
                        ps[0] += f01.x;
                        ps[1] += f01.y;
                        ps[2] += f23.x;
                        ps[3] += f23.y;
                    }
                }
        }
        fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            tma_store_4d(&mg, 0, tx0, ty0, img, sGo);
            bulk_commit();
        }
        // Flush the pool partial when the next tile belongs to another image
        // (or this is the CTA's last tile): fixed-order reduction.
        const int tn = t + static_cast<int>(gridDim.x);
        if (tn >= total || tn / per_img != img) {
#pragma unroll
            for (int i = 0; i < 4; ++i) sRed[(slot * 2 + half) * D + cg * 4 + i] = ps[i];
            __syncthreads();
            for (int c = tid; c < D; c += kAThreads) {
                float sum = 0.f;
                for (int l = 0; l < 2 * G::SLOTS; ++l) sum += sRed[l * D + c];
                sPart[img * D + c] += sum;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) ps[i] = 0.f;
            __syncthreads();
        }
    }
    if (tid == 0) bulk_wait0();
    __syncthreads();
    for (int i = tid; i < p.N * D; i += kAThreads) {
        const int n = i / D, c = i - n * D;
        p.partials[(static_cast<size_t>(n) * gridDim.x + blockIdx.x) * D + c] = sPart[i];
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, G::TMEM_COLS);
}

// ============================== phase B =====================================

// 128 threads (one per tile row) at C <= 32, where four CTAs share an SM;
// 256 at C = 64 (two CTAs per SM): two threads per row (TMEM lane) split its
// columns, halving the serial epilogue work of each thread.
template <int C>
constexpr int b_threads() { return C >= 64 ? 256 : 128; }

template <int C, int D, int F>
__global__ void __launch_bounds__(b_threads<C>(), 1)
    fused_b_kernel(const __grid_constant__ FusedBParams p, const __grid_constant__ CUtensorMap mg,
                   const __grid_constant__ CUtensorMap mx, const __grid_constant__ CUtensorMap mo) {
    using G = GeoB<C, D, F>;
    if (threadIdx.x == 0) {
        prefetch_tmap(&mg);
        prefetch_tmap(&mx);
        prefetch_tmap(&mo);
    }
    constexpr int kTh = b_threads<C>();
    constexpr int kH = kTh / 128;  // threads per tile row
    constexpr int CC = C / kH, DC = D / kH, FC = F / kH;  // columns per thread
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    uint8_t* sG = smem;                  // [128][D] swizzled (span 2D)
    uint8_t* sX = sG + G::G_BYTES;       // [128][C] swizzled (span 2C)
    uint8_t* sA2 = sX + G::X_BYTES;      // LN2(y)
    uint8_t* sO = sA2;                   // output staging: LN2(y) is dead once conv4 has read it
    uint8_t* sA3 = sA2 + G::X_BYTES;     // gated FFN (span 2F)
    uint8_t* sW3 = sA3 + G::A3_BYTES;
    uint8_t* sW4 = sW3 + G::W3_BYTES;
    uint8_t* sW5 = sW4 + G::W4_BYTES;
    float* sB3 = reinterpret_cast<float*>(sW5 + G::W5_BYTES);
    float* sBeta = sB3 + C;
    float* sLw = sBeta + C;
    float* sLb = sLw + C;
    float* sB5 = sLb + C;
    float* sGam = sB5 + C;
    float* sB4 = sGam + C;      // [2F]
    float* sS = sB4 + 2 * F;    // SCA scale [8][D]
    __shared__ uint64_t bar_w, bar_ld, bar_mma;
    __shared__ uint32_t tslot;
    __shared__ int s_fail;
    __shared__ float2 s_stat[2][128];  // kH == 2: per-half (mean, M2) of each row

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r = (warp & 3) * 32 + lane;  // tile row == TMEM lane
    const int hf = warp >> 2;              // column half (0 when one thread owns the row)
    const int tiles = (p.M + 127) / 128;
    const int nimg = (p.M + p.hw - 1) / p.hw;
    for (int i = tid; i < C; i += kTh) {
        sB3[i] = p.b3[i];
        sBeta[i] = p.beta[i];
        sLw[i] = p.ln_w[i];
        sLb[i] = p.ln_b[i];
        sB5[i] = p.b5[i];
        sGam[i] = p.gamma[i];
    }
    for (int i = tid; i < 2 * F; i += kTh) sB4[i] = p.b4[i];
    if (warp == 0) {
        tmem_alloc(&tslot, G::TMEM_COLS);
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(&bar_w, 1);
        mbar_init(&bar_ld, 1);
        mbar_init(&bar_mma, 1);
        s_fail = 0;
        fence_mbar_init();
        mbar_arrive_expect_tx(&bar_w, G::W3_BYTES + G::W4_BYTES + G::W5_BYTES);
        if (p.s) bulk_g2s(sW3, p.w3, G::W3_BYTES, &bar_w);  // else written by the SCA kernel: after the wait
        bulk_g2s(sW4, p.w4, G::W4_BYTES, &bar_w);
        bulk_g2s(sW5, p.w5, G::W5_BYTES, &bar_w);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    pdl_trigger();  // only once this CTA holds its TMEM columns
    const uint64_t d3a = sdesc_kmajor_sw(smem_u32(sG), 2 * D), d3b = sdesc_kmajor(smem_u32(sW3), 128, (D / 8) * 128);
    const uint64_t d4a = sdesc_kmajor_sw(smem_u32(sA2), 2 * C), d4b = sdesc_kmajor(smem_u32(sW4), 128, (C / 8) * 128);
    const uint64_t d5a = sdesc_kmajor_sw(smem_u32(sA3), 2 * F), d5b = sdesc_kmajor(smem_u32(sW5), 128, (F / 8) * 128);
    pdl_wait();  // g, x and the SCA scale (or the SCA-scaled w3) come from earlier kernels
    if (p.s) {
        for (int i = tid; i < nimg * D; i += kTh) sS[i] = p.s[i];
    } else if (tid == 0) {
        bulk_g2s(sW3, p.w3, G::W3_BYTES, &bar_w);
    }
    if (tid == 0 && blockIdx.x < tiles) {
        mbar_arrive_expect_tx(&bar_ld, G::G_BYTES + G::X_BYTES);
        tma_load_2d(sG, &mg, 0, blockIdx.x * 128, &bar_ld);
        tma_load_2d(sX, &mx, 0, blockIdx.x * 128, &bar_ld);
    }
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const bool ok = __syncthreads_and(wait_bar(&bar_w, 0, p.err, 0x40)) != 0;
    uint32_t mma_phase = 0;
    auto mma_wait = [&](uint32_t site) {
        if (!wait_bar(&bar_mma, mma_phase & 1, p.err, site)) s_fail = 1;
        ++mma_phase;
        tc_fence_after();
    };

    int it = 0;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++it) {
        const int m0 = t * 128;
        const int row = m0 + r;
        const int img = row < p.M ? row / p.hw : 0;
        if (!wait_bar(&bar_ld, it & 1, p.err, 0x41)) s_fail = 1;
        __syncthreads();
        if (s_fail) break;
        // SCA: g *= s in place (this thread's half of the row), unless the
        // scale is folded into w3.
        if (p.s) {
            const float* sc = sS + img * D;
#pragma unroll
            for (int q = hf * (DC / 8); q < (hf + 1) * (DC / 8); ++q) {
                uint4* ptr = reinterpret_cast<uint4*>(sG + sw_offset(r, q, 2 * D));
                float f[8];
                h8_to_f(*ptr, f);
#pragma unroll
                for (int i = 0; i < 8; ++i) f[i] *= sc[8 * q + i];
                *ptr = f_to_h8(f);
            }
        }
        fence_async_smem();
        if (tid == 0) bulk_wait_read0();  // the previous output tile has left sO (= sA2, written below)
        __syncthreads();
        if (tid == 0) {  // conv3: [128 x D] x [D -> C]
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < D / 16; ++k)
                mma_f16(tmem, desc_add(d3a, k * 32), desc_add(d3b, k * 256), idesc_f16_f32(128, C), k > 0 ? 1u : 0u);
            mma_commit(&bar_mma);
        }
        mma_wait(0x42);
        // y = x + beta * (acc + b3) (this thread's columns), then LayerNorm2(y) -> A of conv4.
        float y[CC];
        const int cb = hf * CC;
#pragma unroll
        for (int c0 = 0; c0 < CC; c0 += 16) {
            float v[16];
            tmem_ld16(lane_base + cb + c0, v);
            tmem_ld_wait();
#pragma unroll
            for (int g2 = 0; g2 < 2; ++g2) {
                float xv[8];
                h8_to_f(*reinterpret_cast<const uint4*>(sX + sw_offset(r, ((cb + c0) >> 3) + g2, 2 * C)), xv);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int cl = c0 + 8 * g2 + i, c = cb + cl;
                    // round to fp16 like the stored mid-block tensor of the reference
                    y[cl] = __half2float(__float2half(xv[i] + sBeta[c] * (v[8 * g2 + i] + sB3[c])));
                }
            }
        }
        {
            float s1 = 0.f;
#pragma unroll
            for (int c = 0; c < CC; ++c) s1 += y[c];
            float mean = s1 * (1.0f / CC);
            float m2 = 0.f;
#pragma unroll
            for (int c = 0; c < CC; ++c) m2 += (y[c] - mean) * (y[c] - mean);
            if (kH == 2) {  // merge the two halves of the row (Chan's formula)
                s_stat[hf][r] = make_float2(mean, m2);
                __syncthreads();
                const float2 o = s_stat[hf ^ 1][r];
                const float d = mean - o.x;
                mean = 0.5f * (mean + o.x);
                m2 = m2 + o.y + d * d * (0.25f * C);
            }
            const float rstd = rsqrtf(m2 * (1.0f / C) + 1e-6f);
#pragma unroll
            for (int q = 0; q < CC / 8; ++q) {
                float f[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int c = cb + 8 * q + i;
                    f[i] = (y[8 * q + i] - mean) * rstd * sLw[c] + sLb[c];
                }
                *reinterpret_cast<uint4*>(sA2 + sw_offset(r, (cb >> 3) + q, 2 * C)) = f_to_h8(f);
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            // g and x of this tile are consumed: prefetch the next tile.
            if (t + static_cast<int>(gridDim.x) < tiles) {
                const int nm = (t + gridDim.x) * 128;
                mbar_arrive_expect_tx(&bar_ld, G::G_BYTES + G::X_BYTES);
                tma_load_2d(sG, &mg, 0, nm, &bar_ld);
                tma_load_2d(sX, &mx, 0, nm, &bar_ld);
            }
            tc_fence_after();  // conv4: [128 x C] x [C -> 2F]
#pragma unroll
            for (int k = 0; k < C / 16; ++k)
                mma_f16(tmem, desc_add(d4a, k * 32), desc_add(d4b, k * 256), idesc_f16_f32(128, 2 * F),
                        k > 0 ? 1u : 0u);
            mma_commit(&bar_mma);
        }
        mma_wait(0x43);
        // SimpleGate -> A of conv5 (this thread's gate channels).
        const int fb = hf * FC;
#pragma unroll 1
        for (int c0 = fb; c0 < fb + FC; c0 += 16) {
            float va[16], vb[16];
            tmem_ld16(lane_base + c0, va);
            tmem_ld16(lane_base + F + c0, vb);
            tmem_ld_wait();
#pragma unroll
            for (int g2 = 0; g2 < 2; ++g2) {
                float f[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int c = c0 + 8 * g2 + i;
                    f[i] = (va[8 * g2 + i] + sB4[c]) * (vb[8 * g2 + i] + sB4[F + c]);
                }
                *reinterpret_cast<uint4*>(sA3 + sw_offset(r, (c0 >> 3) + g2, 2 * F)) = f_to_h8(f);
            }
        }
        fence_async_smem();
        tc_fence_before();
        if (tid == 0) bulk_wait_read0();  // the previous output tile has left sO
        __syncthreads();
        if (tid == 0) {  // conv5: [128 x F] x [F -> C]
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < F / 16; ++k)
                mma_f16(tmem, desc_add(d5a, k * 32), desc_add(d5b, k * 256), idesc_f16_f32(128, C), k > 0 ? 1u : 0u);
            mma_commit(&bar_mma);
        }
        mma_wait(0x44);
        // out = y + gamma * (acc + b5)
#pragma unroll
        for (int c0 = 0; c0 < CC; c0 += 16) {
            float v[16];
            tmem_ld16(lane_base + cb + c0, v);
            tmem_ld_wait();
#pragma unroll
            for (int g2 = 0; g2 < 2; ++g2) {
                float f[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int cl = c0 + 8 * g2 + i, c = cb + cl;
                    f[i] = y[cl] + sGam[c] * (v[8 * g2 + i] + sB5[c]);
                }
                *reinterpret_cast<uint4*>(sO + sw_offset(r, ((cb + c0) >> 3) + g2, 2 * C)) = f_to_h8(f);
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tma_store_2d(&mo, 0, m0, sO);
            bulk_commit();
        }
    }
    if (tid == 0) bulk_wait0();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, G::TMEM_COLS);
}

// ============================== host ========================================

}  // namespace

int encode_f16_map(CUtensorMap* m, int rank, const void* base, const cuuint64_t* dims, const cuuint64_t* strides,
                   const cuuint32_t* box, CUtensorMapSwizzle swz) {
    auto fn = tensor_map_encoder();
    if (!fn) return dn_fail(DN_ERR_CUDA, "fused: cuTensorMapEncodeTiled unavailable");
    cuuint32_t es[5] = {1, 1, 1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank, const_cast<void*>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return dn_fail_str(DN_ERR_CUDA, "fused: cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
    return DN_OK;
}

int sm_count() {
    static int n = 0;
    if (!n) {
        int d = 0;
        cudaGetDevice(&d);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
        if (n <= 0) n = 148;
    }
    return n;
}

namespace {

CUtensorMapSwizzle swz_for(int bytes) {
    return bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
}

template <int C, int D>
int run_a(const FusedAParams& p, int grid, cudaStream_t s) {
    using G = GeoA<C, D>;
    auto kern = fused_a_kernel<C, D>;
    static bool cfg = false;
    if (!cfg) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM);
        if (e != cudaSuccess) return dn_cuda_fail(e, "fused_a: smem attribute");
        cfg = true;
    }
    CUtensorMap mx, mg;
    const cuuint64_t dx[4] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(p.W), static_cast<cuuint64_t>(p.H),
                              static_cast<cuuint64_t>(p.N)};
    const cuuint64_t sx[3] = {static_cast<cuuint64_t>(C) * 2, static_cast<cuuint64_t>(p.W) * C * 2,
                              static_cast<cuuint64_t>(p.H) * p.W * C * 2};
    const cuuint32_t bx[4] = {static_cast<cuuint32_t>(C), G::WW, G::HH, 1};
    int rc = encode_f16_map(&mx, 4, p.x, dx, sx, bx, swz_for(2 * C));
    if (rc != DN_OK) return rc;
    const cuuint64_t dg[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(p.W), static_cast<cuuint64_t>(p.H),
                              static_cast<cuuint64_t>(p.N)};
    const cuuint64_t sg[3] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(p.W) * D * 2,
                              static_cast<cuuint64_t>(p.H) * p.W * D * 2};
    const cuuint32_t bg[4] = {static_cast<cuuint32_t>(D), G::TW, G::TH, 1};
    rc = encode_f16_map(&mg, 4, p.g, dg, sg, bg, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != DN_OK) return rc;
    cudaError_t e = launch_pdl(kern, dim3(grid), dim3(kAThreads), G::SMEM, s, p, mx, mg);
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "fused_a: launch");
}

template <int C, int D, int F>
int run_b(const FusedBParams& p, cudaStream_t s) {
    using G = GeoB<C, D, F>;
    auto kern = fused_b_kernel<C, D, F>;
    static bool cfg = false;
    if (!cfg) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM);
        if (e != cudaSuccess) return dn_cuda_fail(e, "fused_b: smem attribute");
        cfg = true;
    }
    CUtensorMap mg, mx, mo;
    const cuuint32_t bD[2] = {static_cast<cuuint32_t>(D), 128};
    const cuuint32_t bC[2] = {static_cast<cuuint32_t>(C), 128};
    const cuuint64_t dG[2] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(p.M)};
    const cuuint64_t dC[2] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(p.M)};
    const cuuint64_t sG[1] = {static_cast<cuuint64_t>(D) * 2};
    const cuuint64_t sC[1] = {static_cast<cuuint64_t>(C) * 2};
    int rc = encode_f16_map(&mg, 2, p.g, dG, sG, bD, swz_for(2 * D));
    if (rc == DN_OK) rc = encode_f16_map(&mx, 2, p.x, dC, sC, bC, swz_for(2 * C));
    if (rc == DN_OK) rc = encode_f16_map(&mo, 2, p.out, dC, sC, bC, swz_for(2 * C));
    if (rc != DN_OK) return rc;
    const int tiles = (p.M + 127) / 128;
    const int per_sm = std::max(1, std::min(512 / G::TMEM_COLS, (227 * 1024) / (G::SMEM + 2048)));
    const int grid = std::min(tiles, sm_count() * per_sm);
    cudaError_t e = launch_pdl(kern, dim3(grid), dim3(b_threads<C>()), G::SMEM, s, p, mg, mx, mo);
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "fused_b: launch");
}

}  // namespace

bool fused_supported(int C, int D, int F) {
    return (C == 16 && D == 16 && (F == 16 || F == 32)) || (C == 32 && D == 32 && (F == 32 || F == 64)) ||
           (C == 64 && D == 64 && F == 64);
}

int fused_a_grid(int C, int D, int N, int H, int W) {
    auto geo = [&](int TH, int TW, int smem, int cols) {
        const int tiles = N * ((H + TH - 1) / TH) * ((W + TW - 1) / TW);
        const int per_sm = std::max(1, std::min(512 / cols, (227 * 1024) / (smem + 2048)));
        return std::max(1, std::min(tiles, sm_count() * per_sm));
    };
    if (C == 16) return geo(GeoA<16, 16>::TH, GeoA<16, 16>::TW, GeoA<16, 16>::SMEM, GeoA<16, 16>::TMEM_COLS);
    if (C == 32) return geo(GeoA<32, 32>::TH, GeoA<32, 32>::TW, GeoA<32, 32>::SMEM, GeoA<32, 32>::TMEM_COLS);
    return geo(GeoA<64, 64>::TH, GeoA<64, 64>::TW, GeoA<64, 64>::SMEM, GeoA<64, 64>::TMEM_COLS);
}

int launch_fused_a(const FusedAParams& p, int C, int D, int grid, cudaStream_t s) {
    if (p.N > 8) return dn_fail(DN_ERR_UNSUPPORTED, "fused_a: batch > 8");
    if (C == 16 && D == 16) return run_a<16, 16>(p, grid, s);
    if (C == 32 && D == 32) return run_a<32, 32>(p, grid, s);
    if (C == 64 && D == 64) return run_a<64, 64>(p, grid, s);
    return dn_fail(DN_ERR_UNSUPPORTED, "fused_a: channel configuration");
}

int launch_fused_b(const FusedBParams& p, int C, int D, int F, cudaStream_t s) {
    if ((p.M + p.hw - 1) / p.hw > 8) return dn_fail(DN_ERR_UNSUPPORTED, "fused_b: batch > 8");
    if (C == 16 && D == 16 && F == 16) return run_b<16, 16, 16>(p, s);
    if (C == 16 && D == 16 && F == 32) return run_b<16, 16, 32>(p, s);
    if (C == 32 && D == 32 && F == 32) return run_b<32, 32, 32>(p, s);
    if (C == 32 && D == 32 && F == 64) return run_b<32, 32, 64>(p, s);
    if (C == 64 && D == 64 && F == 64) return run_b<64, 64, 64>(p, s);
    return dn_fail(DN_ERR_UNSUPPORTED, "fused_b: channel configuration");
}

}  // namespace dnb
