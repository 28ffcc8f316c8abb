// Stand-alone convolution layers as one fused implicit GEMM each:
// DeformConv2dLayer (modulated deformable convolution, DCNv2) and
// Conv2dLayer (regular convolution with any kernel, padding, stride,
// dilation and groups).
//
// Deformable:
//   out[n, o, y, x] = bias[o] + sum_{g, k, c} W[o, g*cpg + c, k] *
//                     bilinear(in[n, g*cpg + c], p(y, x, k) + off[n, g, k]) * sigmoid(mask[n, g, k])
//
// The reference (DeformConv2dLayer::forward, src/layers/deform_conv2d.cu
// :105-184) materialises the whole modulated im2col matrix
// (deform_im2col_kernel, src/kernels/deform_im2col.cuh:78-142; Cin*9 x N*H*W
// FP16, ~2.4 GB for 64 channels at 1088x1920) and multiplies it with a
// FP16-accumulating cublasHgemm. Here one CTA owns a stream of 128-pixel
// tiles; per 64-wide K chunk:
//   * CUDA-core threads build the modulated A tile in shared memory, one
//     work item per (pixel, deform group, tap): the sample point, the four
//     corner weights and the sigmoid of the mask are computed once and reused
//     for the group's cpg channels, which are gathered as vectors from an
//     NHWC copy of the input; values are rounded to FP16 as the reference's
//     im2col buffer is;
//   * the B chunk (weights, K order (group, tap, channel)) arrives by bulk
//     copy; one thread issues tcgen05.mma (M = 128, N = Cout, FP32 in TMEM);
//   * two stages double-buffer A and B so sampling overlaps the MMA.
// The epilogue adds the bias and writes NCHW (consecutive lanes = consecutive
// pixels of one output plane). Sampling rule (bilinear_sample,
// deform_im2col.cuh:34-69): zero when h < -1, h > H, w < -1 or w > W;
// corners outside the image contribute zero.
//
// Regular (Conv2dLayer::forward, src/layers/conv2d.cu:94-150, a cuDNN
// convolution plus a bias pass in the reference): the same kernel with
// integer sample points, so an A-tile item is one vector copy from the NHWC
// input (zero outside the image). K runs over (block of cpg input channels,
// tap, channel); a grouped convolution packs B block-diagonally (weights of
// input channels outside an output's group are zero), and more than 256
// output channels run as 256-wide slabs over the same NHWC copy.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "capi_internal.h"
#include "conv_internal.h"
#include "denoiser_b200_layers.h"
#include "launch.cuh"
#include "sm100.cuh"
#include "status.h"

namespace dnb {
namespace {

constexpr int kThreads = 256;
constexpr int kKC = 64;                   // K chunk (one 128-byte swizzled row)
constexpr int kABytes = 128 * kKC * 2;    // 16 KB

// Output modes of the epilogue.
enum : int {
    kOutNCHW = 0,  // out[n][o][y][x]
    kOutNHWC = 1,  // out[n][y][x][o] (a feature map that a later conv reads without a transpose)
    kOutFuse = 2,  // no activation store: the 1x1 fusion of the output channels (below)
};

struct DcnParams {
    const __half* xt;    // input, NHWC [N][H][W][Cin]
    const __half* off;   // [N][2*dg*KK][Ho][Wo] (dy, dx per (group, tap))
    const __half* msk;   // [N][dg*KK][Ho][Wo] (pre-sigmoid)
    const __half* off2;  // optional second term of the offsets (same layout; summed in FP32), or null
    const __half* msk2;  // optional second term of the raw masks, or null
    __half* out;         // kOutNCHW: [N][Cout][Ho][Wo]; kOutNHWC: [N][Ho][Wo][Cout]
    int out_mode;
    // kOutFuse (batch 1): fuse_acc[j][pix] += sum_o fuse_w[j][o] * (acc[o] + bias[o]) for j < 3
    // (FP32 planes); with fuse_out set, the sum is written there as FP16 NCHW planes instead.
    const float* fuse_w;   // [3][NT]
    float* fuse_acc;       // [3][Ho*Wo]
    __half* fuse_out;      // [3][Ho*Wo] or null
    const uint8_t* bpack;  // [k_chunks][NT x 64] no-swizzle K-major tiles (this launch's output slab)
    const float* bias;     // [NT] (zero padded)
    int N, H, W, Ho, Wo, Cin, Cout;
    int cout_base;         // first output channel of this launch's slab
    int kw, KK, pad, stride, dil, dg, cpg, k_chunks;
    uint32_t* err;
};

// cpg channels of one corner, VEC channels per load (VEC in {1, 2, 4, 8}).
template <int VEC>
struct Vec;
template <>
struct Vec<8> {
    using T = uint4;
};
template <>
struct Vec<4> {
    using T = uint2;
};
template <>
struct Vec<2> {
    using T = uint32_t;
};
template <>
struct Vec<1> {
    using T = uint16_t;
};

template <int VEC>
__device__ __forceinline__ void unpack_vec(const typename Vec<VEC>::T& v, float (&f)[VEC]) {
    if constexpr (VEC == 8) {
        h8_to_f(v, f);
    } else if constexpr (VEC == 4) {
        const float2 a = unpack_half2(v.x), b = unpack_half2(v.y);
        f[0] = a.x;
        f[1] = a.y;
        f[2] = b.x;
        f[3] = b.y;
    } else if constexpr (VEC == 2) {
        const float2 a = unpack_half2(v);
        f[0] = a.x;
        f[1] = a.y;
    } else {
        __half h;
        memcpy(&h, &v, 2);
        f[0] = __half2float(h);
    }
}

template <int VEC>
__device__ __forceinline__ typename Vec<VEC>::T pack_vec(const float (&f)[VEC]) {
    typename Vec<VEC>::T v;
    if constexpr (VEC == 8) {
        v = f_to_h8(f);
    } else if constexpr (VEC == 4) {
        v = make_uint2(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]));
    } else if constexpr (VEC == 2) {
        v = pack_half2(f[0], f[1]);
    } else {
        const __half h = __float2half(f[0]);
        memcpy(&v, &h, 2);
    }
    return v;
}

// DEFORM: modulated deformable sampling. Otherwise a regular convolution:
// the sample points are integer, so each item copies one vector of the NHWC
// input (zero outside the image = zero padding); `dg` then counts blocks of
// `cpg` input channels and B is block-diagonal for grouped convolutions.
// Two CTAs per SM (at most ~100 KB of shared memory and 256 TMEM columns
// each): the A-tile builders of one CTA wait on global loads while the other
// CTA's run.
template <int NT, int VEC, bool DEFORM>
__global__ void __launch_bounds__(kThreads, 2) conv_kernel(const __grid_constant__ DcnParams p) {
    constexpr int kBBytes = NT * kKC * 2;
    constexpr uint32_t kCols = NT < 32 ? 32 : NT;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sA[2] = {smem, smem + kABytes};
    uint8_t* sB[2] = {smem + 2 * kABytes, smem + 2 * kABytes + kBBytes};
    float* sBias = reinterpret_cast<float*>(smem + 2 * kABytes + 2 * kBBytes);
    __shared__ uint64_t bar_b[2], bar_mma[2];
    __shared__ float sFuse[3][128];  // kOutFuse: the second column half's partial sums per tile row
    // Per (group/block, tap) combo: the channel offset g * cpg and the tap's
    // row / column offsets (ki * dil, kj * dil), for the batched A builders.
    constexpr int kMaxCombos = 512;
    __shared__ int2 sCombo[kMaxCombos];
    __shared__ uint32_t tslot;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < NT; i += kThreads) sBias[i] = p.bias[i];
    const int n_combos = p.dg * p.KK;
    for (int gk = tid; gk < n_combos && gk < kMaxCombos; gk += kThreads) {
        const int g = gk / p.KK, k = gk - g * p.KK;
        const int ki = k / p.kw, kj = k - ki * p.kw;
        sCombo[gk] = make_int2(g * p.cpg, (ki * p.dil) | ((kj * p.dil) << 16));
    }
    if (warp == 0) {
        tmem_alloc(&tslot, kCols);
        tmem_relinquish();
    }
    if (tid == 0) {
        for (int s = 0; s < 2; ++s) {
            mbar_init(&bar_b[s], 1);
            mbar_init(&bar_mma[s], 1);
        }
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    pdl_trigger();  // only once this CTA holds its TMEM columns
    pdl_wait();

    const int HWo = p.Ho * p.Wo;
    const int M = p.N * HWo;
    const int tiles = (M + 127) / 128;
    const int combos = p.dg * p.KK;
    const int cpc = kKC / p.cpg;  // (group, tap) combos per K chunk
    const uint32_t idesc = idesc_f16_f32(128, NT);
    int it = 0;  // chunk counter across tiles (stage = it & 1, use = it >> 1)
    bool ok = true;
    // The batched builders index with 32-bit element offsets and the combo
    // table: they run when every tensor they index has < 2^31 elements.
    const bool fast = n_combos <= kMaxCombos &&
                      static_cast<long long>(p.N) * p.H * p.W * p.Cin < (1LL << 31) &&
                      (!DEFORM || static_cast<long long>(p.N) * 2 * n_combos * HWo < (1LL << 31));
    for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        // Pixel coordinates of this thread's rows of the tile (batched builders):
        // regular: rows tid / 8 + 32 u; deformable: row tid % 128.
        int py[4], px[4], pn[4];
        bool pok[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int r = DEFORM ? (tid & 127) : (tid >> 3) + 32 * u;
            const int m = tile * 128 + r;
            pok[u] = m < M;
            const int n = pok[u] ? m / HWo : 0;
            const int pix = pok[u] ? m - n * HWo : 0;
            const int ho = pix / p.Wo, wo = pix - ho * p.Wo;
            py[u] = ho * p.stride - p.pad;
            px[u] = wo * p.stride - p.pad;
            pn[u] = DEFORM ? pix : n * p.H;  // deformable: keep the plane index; n below
        }
        const int dn = DEFORM && pok[0] ? (tile * 128 + (tid & 127)) / HWo : 0;  // image of the deformable row
        for (int j = 0; j < p.k_chunks; ++j, ++it) {
            const int s = it & 1;
            const uint32_t use = static_cast<uint32_t>(it >> 1);
            // Stage free: the MMA that read it two chunks ago has completed.
            bool waited = true;
            if (use > 0) waited = mbar_wait(&bar_mma[s], (use - 1) & 1u);
            if (!__syncthreads_and(waited)) {
                if (tid == 0) report_error(p.err, 0x60, kErrMbarTimeout);
                ok = false;
                break;
            }
            if (tid == 0) {
                mbar_arrive_expect_tx(&bar_b[s], kBBytes);
                bulk_g2s(sB[s], p.bpack + static_cast<size_t>(j) * kBBytes, kBBytes, &bar_b[s]);
            }
            // A tile of chunk j. The common shapes take batched paths that put
            // all of a thread's loads in flight before any is used (one memory
            // latency per chunk instead of one or two per item):
            bool built = false;
            if constexpr (!DEFORM && VEC == 8) {
                if (fast) {
                    // Regular conv, 8-channel vectors: 128 pixels x 8 vectors; thread
                    // tid takes vector kv = tid % 8 of pixels tid / 8 + 32 u, so a
                    // warp reads 4 pixels x 128 contiguous bytes.
                    const int kv = tid & 7;
                    const int kk = kv * 8, lc = kk / p.cpg, v0 = kk - lc * p.cpg;
                    const int gk = j * cpc + lc;
                    const int2 cb = gk < combos ? sCombo[gk] : make_int2(0, 0);
                    const int oy = cb.y & 0xFFFF, ox = cb.y >> 16;
                    uint4 v[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int yy = py[u] + oy, xx = px[u] + ox;
                        v[u] = make_uint4(0u, 0u, 0u, 0u);
                        if (pok[u] && gk < combos && yy >= 0 && yy < p.H && xx >= 0 && xx < p.W)
                            v[u] = *reinterpret_cast<const uint4*>(p.xt + (((pn[u] + yy) * p.W + xx) * p.Cin + cb.x + v0));
                    }
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        *reinterpret_cast<uint4*>(sA[s] + sw_offset((tid >> 3) + 32 * u, kv, 128)) = v[u];
                    built = true;
                }
            }
            if constexpr (DEFORM && VEC == 8) {
                if (p.cpg == 8 && fast) {
                    // Deformable, 8 channels per group: 8 (group, tap) combos per
                    // chunk; thread tid samples pixel tid % 128 for combos
                    // tid / 128 + 2 u: offsets and masks of all four first, then
                    // all 16 corner vectors, then the blends (packed fp32).
                    const int r = tid & 127;
                    const int pix = pn[0];
                    float dy[4], dx[4], raw[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int gk = j * cpc + (tid >> 7) + 2 * u;
                        dy[u] = dx[u] = raw[u] = 0.f;
                        if (pok[0] && gk < combos) {
                            const int ob = (dn * 2 * combos + 2 * gk) * HWo + pix;
                            const int mb = (dn * combos + gk) * HWo + pix;
                            dy[u] = __half2float(p.off[ob]);
                            dx[u] = __half2float(p.off[ob + HWo]);
                            raw[u] = __half2float(p.msk[mb]);
                            if (p.off2) {  // offsets and masks given as two terms (uniform branch)
                                dy[u] += __half2float(p.off2[ob]);
                                dx[u] += __half2float(p.off2[ob + HWo]);
                                raw[u] += __half2float(p.msk2[mb]);
                            }
                        }
                    }
                    uint4 cv[4][4];
                    float cw[4][4];
                    const __half* base = p.xt + static_cast<size_t>(dn) * p.H * p.W * p.Cin;
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int gk = j * cpc + (tid >> 7) + 2 * u;
                        const int2 cb = gk < combos ? sCombo[gk] : make_int2(0, 0);
                        const float hs = static_cast<float>(py[0] + (cb.y & 0xFFFF)) + dy[u];
                        const float ws = static_cast<float>(px[0] + (cb.y >> 16)) + dx[u];
                        const bool in = pok[0] && gk < combos &&
                                        !(hs < -1.f || hs > static_cast<float>(p.H) || ws < -1.f || ws > static_cast<float>(p.W));
                        const int h0 = in ? static_cast<int>(floorf(hs)) : 0, w0 = in ? static_cast<int>(floorf(ws)) : 0;
                        const float dh = hs - static_cast<float>(h0), dw = ws - static_cast<float>(w0);
                        const float wq[4] = {(1.f - dh) * (1.f - dw), (1.f - dh) * dw, dh * (1.f - dw), dh * dw};
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const int yy = h0 + (q >> 1), xx = w0 + (q & 1);
                            cv[u][q] = make_uint4(0u, 0u, 0u, 0u);
                            cw[u][q] = 0.f;
                            if (in && yy >= 0 && yy < p.H && xx >= 0 && xx < p.W) {
                                cv[u][q] = *reinterpret_cast<const uint4*>(base + ((yy * p.W + xx) * p.Cin + cb.x));
                                cw[u][q] = wq[q];
                            }
                        }
                    }
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float mask = 1.f / (1.f + expf(-raw[u]));
                        const uint32_t c0[4] = {cv[u][0].x, cv[u][0].y, cv[u][0].z, cv[u][0].w};
                        const uint32_t c1[4] = {cv[u][1].x, cv[u][1].y, cv[u][1].z, cv[u][1].w};
                        const uint32_t c2[4] = {cv[u][2].x, cv[u][2].y, cv[u][2].z, cv[u][2].w};
                        const uint32_t c3[4] = {cv[u][3].x, cv[u][3].y, cv[u][3].z, cv[u][3].w};
                        const float2 w0 = make_float2(cw[u][0], cw[u][0]), w1 = make_float2(cw[u][1], cw[u][1]);
                        const float2 w2 = make_float2(cw[u][2], cw[u][2]), w3 = make_float2(cw[u][3], cw[u][3]);
                        const float2 mk = make_float2(mask, mask), z = make_float2(0.f, 0.f);
                        uint32_t o[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            float2 t = ffma2(unpack_half2(c0[i]), w0, z);
                            t = ffma2(unpack_half2(c1[i]), w1, t);
                            t = ffma2(unpack_half2(c2[i]), w2, t);
                            t = ffma2(unpack_half2(c3[i]), w3, t);
                            t = ffma2(t, mk, z);
                            o[i] = pack_half2(t.x, t.y);
                        }
                        *reinterpret_cast<uint4*>(sA[s] + sw_offset(r, (tid >> 7) + 2 * u, 128)) =
                            make_uint4(o[0], o[1], o[2], o[3]);
                    }
                    built = true;
                }
            }
            // Other shapes: item = (pixel r, combo lc), one at a time.
            for (int item = built ? 128 * cpc : tid; item < 128 * cpc; item += kThreads) {
                const int r = item & 127;
                const int lc = item >> 7;
                const int gk = j * cpc + lc;
                const int m = tile * 128 + r;
                float wts[4] = {0.f, 0.f, 0.f, 0.f};
                const __half* corner[4] = {nullptr, nullptr, nullptr, nullptr};
                if (!DEFORM && m < M && gk < combos) {
                    const int n = m / HWo;
                    const int pix = m - n * HWo;
                    const int ho = pix / p.Wo, wo = pix - ho * p.Wo;
                    const int g = gk / p.KK, k = gk - g * p.KK;
                    const int ki = k / p.kw, kj = k - ki * p.kw;
                    const int yy = ho * p.stride - p.pad + ki * p.dil;
                    const int xx = wo * p.stride - p.pad + kj * p.dil;
                    const bool in = yy >= 0 && yy < p.H && xx >= 0 && xx < p.W;
                    const __half* src =
                        p.xt + ((static_cast<size_t>(n) * p.H + (in ? yy : 0)) * p.W + (in ? xx : 0)) * p.Cin + g * p.cpg;
                    for (int v0 = 0; v0 < p.cpg; v0 += VEC) {
                        typename Vec<VEC>::T v{};
                        if (in) v = *reinterpret_cast<const typename Vec<VEC>::T*>(src + v0);
                        const int kk = lc * p.cpg + v0;
                        *reinterpret_cast<typename Vec<VEC>::T*>(sA[s] + sw_offset(r, kk >> 3, 128) + (kk & 7) * 2) = v;
                    }
                    continue;
                }
                if (DEFORM && m < M && gk < combos) {
                    const int n = m / HWo;
                    const int pix = m - n * HWo;
                    const int ho = pix / p.Wo, wo = pix - ho * p.Wo;
                    const int g = gk / p.KK, k = gk - g * p.KK;
                    const int ki = k / p.kw, kj = k - ki * p.kw;
                    const size_t ob = (static_cast<size_t>(n) * 2 * combos + 2 * gk) * HWo + pix;
                    const size_t mb = (static_cast<size_t>(n) * combos + gk) * HWo + pix;
                    float dy = __half2float(p.off[ob]);
                    float dx = __half2float(p.off[ob + HWo]);
                    float raw = __half2float(p.msk[mb]);
                    if (p.off2) {  // offsets and masks given as two terms (uniform branch)
                        dy += __half2float(p.off2[ob]);
                        dx += __half2float(p.off2[ob + HWo]);
                        raw += __half2float(p.msk2[mb]);
                    }
                    const float mask = 1.f / (1.f + expf(-raw));
                    const float hs = static_cast<float>(ho * p.stride - p.pad + ki * p.dil) + dy;
                    const float ws = static_cast<float>(wo * p.stride - p.pad + kj * p.dil) + dx;
                    if (!(hs < -1.f || hs > static_cast<float>(p.H) || ws < -1.f || ws > static_cast<float>(p.W))) {
                        const int h0 = static_cast<int>(floorf(hs)), w0 = static_cast<int>(floorf(ws));
                        const float dh = hs - static_cast<float>(h0), dw = ws - static_cast<float>(w0);
                        const float cw[4] = {(1.f - dh) * (1.f - dw), (1.f - dh) * dw, dh * (1.f - dw), dh * dw};
                        const __half* base = p.xt + static_cast<size_t>(n) * p.H * p.W * p.Cin + g * p.cpg;
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const int yy = h0 + (q >> 1), xx = w0 + (q & 1);
                            if (yy >= 0 && yy < p.H && xx >= 0 && xx < p.W) {
                                corner[q] = base + (static_cast<size_t>(yy) * p.W + xx) * p.Cin;
                                wts[q] = cw[q];
                            }
                        }
                        for (int v0 = 0; v0 < p.cpg; v0 += VEC) {
                            float acc[VEC];
#pragma unroll
                            for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
                            float vv[4][VEC];
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                if (corner[q]) {
                                    unpack_vec<VEC>(*reinterpret_cast<const typename Vec<VEC>::T*>(corner[q] + v0), vv[q]);
                                } else {
#pragma unroll
                                    for (int e = 0; e < VEC; ++e) vv[q][e] = 0.f;
                                }
                            }
#pragma unroll
                            for (int e = 0; e < VEC; ++e) {
                                const float val = vv[0][e] * wts[0] + vv[1][e] * wts[1] + vv[2][e] * wts[2] +
                                                  vv[3][e] * wts[3];
                                acc[e] = val * mask;
                            }
                            const int kk = lc * p.cpg + v0;  // K offset inside the chunk
                            *reinterpret_cast<typename Vec<VEC>::T*>(sA[s] + sw_offset(r, kk >> 3, 128) +
                                                                     (kk & 7) * 2) = pack_vec<VEC>(acc);
                        }
                        continue;
                    }
                }
                // Zero sample (outside the image, past the last combo, or past the last pixel).
                for (int v0 = 0; v0 < p.cpg; v0 += VEC) {
                    float z[VEC];
#pragma unroll
                    for (int e = 0; e < VEC; ++e) z[e] = 0.f;
                    const int kk = lc * p.cpg + v0;
                    *reinterpret_cast<typename Vec<VEC>::T*>(sA[s] + sw_offset(r, kk >> 3, 128) + (kk & 7) * 2) =
                        pack_vec<VEC>(z);
                }
            }
            fence_async_smem();
            __syncthreads();
            if (tid == 0) {
                if (!mbar_wait(&bar_b[s], use & 1u)) {
                    report_error(p.err, 0x61, kErrMbarTimeout);
                } else {
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA[s]), b0 = smem_u32(sB[s]);
#pragma unroll
                    for (int k = 0; k < kKC / 16; ++k)
                        mma_f16(tmem, sdesc_kmajor_sw(a0 + k * 32, 128), sdesc_kmajor(b0 + k * 256, 128, 1024), idesc,
                                (j > 0 || k > 0) ? 1u : 0u);
                }
                mma_commit(&bar_mma[s]);
            }
        }
        if (!ok) break;
        // Epilogue: all MMAs of the tile are in TMEM once the last commit lands.
        const int sl = (it - 1) & 1;
        const uint32_t ul = static_cast<uint32_t>((it - 1) >> 1);
        if (!__syncthreads_and(mbar_wait(&bar_mma[sl], ul & 1u))) {
            if (tid == 0) report_error(p.err, 0x62, kErrMbarTimeout);
            break;
        }
        tc_fence_after();
        {
            const int q4 = warp & 3;
            const int r = q4 * 32 + lane;
            const int m = tile * 128 + r;
            const int half = warp >> 2;
            const int c_lo = NT >= 32 ? half * (NT / 2) : (half == 0 ? 0 : NT);
            const int c_hi = NT >= 32 ? c_lo + NT / 2 : (half == 0 ? NT : NT);
            const int n = m / HWo, pix = m - n * HWo;
            const int cmax = p.Cout - p.cout_base;  // channels of this slab that exist
            if (p.out_mode == kOutFuse) {
                // 1x1 fusion of this row's output channels into three planes.
                float f3[3] = {0.f, 0.f, 0.f};
                for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
                    float v[16];
                    tmem_ld16(tmem + c0 + (static_cast<uint32_t>(q4 * 32) << 16), v);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        if (c0 + e < cmax) {
                            const float a = v[e] + sBias[c0 + e];
#pragma unroll
                            for (int j = 0; j < 3; ++j) f3[j] = fmaf(p.fuse_w[j * NT + c0 + e], a, f3[j]);
                        }
                    }
                }
                if (half) {
#pragma unroll
                    for (int j = 0; j < 3; ++j) sFuse[j][r] = f3[j];
                }
                __syncthreads();
                if (!half && m < M) {
#pragma unroll
                    for (int j = 0; j < 3; ++j) {
                        const size_t at = static_cast<size_t>(j) * HWo + pix;
                        const float tot = p.fuse_acc[at] + (f3[j] + sFuse[j][r]);
                        if (p.fuse_out)
                            p.fuse_out[at] = __float2half(tot);
                        else
                            p.fuse_acc[at] = tot;
                    }
                }
            } else if (p.out_mode == kOutNHWC) {
                __half* orow = p.out + static_cast<size_t>(m) * p.Cout + p.cout_base;
                for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
                    float v[16];
                    tmem_ld16(tmem + c0 + (static_cast<uint32_t>(q4 * 32) << 16), v);
                    tmem_ld_wait();
                    if (m < M) {
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            if (c0 + e < cmax) orow[c0 + e] = __float2half(v[e] + sBias[c0 + e]);
                    }
                }
            } else {
                __half* orow = p.out + (static_cast<size_t>(n) * p.Cout + p.cout_base) * HWo + pix;
                for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
                    float v[16];
                    tmem_ld16(tmem + c0 + (static_cast<uint32_t>(q4 * 32) << 16), v);
                    tmem_ld_wait();
                    if (m < M) {
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            if (c0 + e < cmax) orow[static_cast<size_t>(c0 + e) * HWo] = __float2half(v[e] + sBias[c0 + e]);
                    }
                }
            }
        }
        tc_fence_before();
        __syncthreads();  // TMEM read before the next tile's first MMA overwrites it
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, kCols);
}

// NCHW -> NHWC, 32 x 32 tiles through shared memory.
__global__ void __launch_bounds__(256) to_nhwc_kernel(const __half* __restrict__ in, __half* __restrict__ out, int C,
                                                      int HW) {
    __shared__ __half t[32][34];
    pdl_trigger();
    pdl_wait();
    const int n = blockIdx.z;
    const int p0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
    const __half* src = in + static_cast<size_t>(n) * C * HW;
    __half* dst = out + static_cast<size_t>(n) * C * HW;
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int c = c0 + i, px = p0 + threadIdx.x;
        if (c < C && px < HW) t[i][threadIdx.x] = src[static_cast<size_t>(c) * HW + px];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int px = p0 + i, c = c0 + threadIdx.x;
        if (c < C && px < HW) dst[static_cast<size_t>(px) * C + c] = t[threadIdx.x][i];
    }
}

int next_pow2(int v) {
    int q = 1;
    while (q < v) q <<= 1;
    return q;
}

}  // namespace
}  // namespace dnb

using namespace dnb;

struct dn_dcn {
    int device = 0;
    int cin = 0, cout = 0, kh = 0, kw = 0, pad = 1, stride = 1, dil = 1, dg = 8, cpg = 0, NT = 0, k_chunks = 0;
    uint8_t* bpack = nullptr;  // device: packed weights
    float* bias = nullptr;     // device: [NT]
    __half* xt = nullptr;      // device: NHWC copy of the input (grown on demand)
    size_t xt_bytes = 0;
    uint32_t* err = nullptr;
};

namespace {

template <int NT, int VEC, bool DEFORM>
int run_conv(const DcnParams& p, int device, cudaStream_t s) {
    constexpr int smem = 1024 + 2 * kABytes + 2 * NT * kKC * 2 + NT * 4;
    static bool configured[64] = {};
    if (device >= 0 && device < 64 && !configured[device]) {
        cudaError_t e = cudaFuncSetAttribute(conv_kernel<NT, VEC, DEFORM>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return dn_cuda_fail(e, "dcn: smem attribute");
        configured[device] = true;
    }
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    const int tiles = (p.N * p.Ho * p.Wo + 127) / 128;
    const int grid = std::max(1, std::min(tiles, 2 * sms));  // two CTAs per SM
    cudaError_t e = launch_pdl(conv_kernel<NT, VEC, DEFORM>, dim3(grid), dim3(kThreads), smem, s, p);
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "conv: launch");
}

template <int NT, bool DEFORM>
int run_conv_vec(const DcnParams& p, int device, cudaStream_t s) {
    if (p.cpg % 8 == 0) return run_conv<NT, 8, DEFORM>(p, device, s);
    if (p.cpg % 4 == 0) return run_conv<NT, 4, DEFORM>(p, device, s);
    if (p.cpg % 2 == 0) return run_conv<NT, 2, DEFORM>(p, device, s);
    return run_conv<NT, 1, DEFORM>(p, device, s);
}

template <bool DEFORM>
int run_conv_nt(const DcnParams& p, int nt, int device, cudaStream_t s) {
    switch (nt) {
        case 16: return run_conv_vec<16, DEFORM>(p, device, s);
        case 32: return run_conv_vec<32, DEFORM>(p, device, s);
        case 64: return run_conv_vec<64, DEFORM>(p, device, s);
        case 128: return run_conv_vec<128, DEFORM>(p, device, s);
        default: return run_conv_vec<256, DEFORM>(p, device, s);
    }
}

struct DevGuard {
    int prev = -1;
    explicit DevGuard(int d) {
        cudaGetDevice(&prev);
        if (prev != d) cudaSetDevice(d);
    }
    ~DevGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace

namespace dnb {

int dcn_build(const float* w, const float* bias, int cout, int cin, int kh, int kw, int pad, int stride, int dilation,
              int deform_groups, int device, dn_dcn** out) {
    *out = nullptr;
    if (pad < 0 || stride <= 0 || dilation <= 0 || deform_groups <= 0 || cout <= 0 || cin <= 0 || kh <= 0 || kw <= 0)
        return dn_fail(DN_ERR_INVALID_ARG, "dn_dcn_create: bad pad/stride/dilation/deform_groups");
    auto L = std::make_unique<dn_dcn>();
    L->device = device;
    L->cout = cout;
    L->cin = cin;
    L->kh = kh;
    L->kw = kw;
    L->pad = pad;
    L->stride = stride;
    L->dil = dilation;
    L->dg = deform_groups;
    if (L->cin % deform_groups != 0)
        return dn_fail(DN_ERR_INVALID_ARG, "dn_dcn_create: in_channels must be divisible by deform_groups");
    L->cpg = L->cin / deform_groups;
    if (kKC % L->cpg != 0) return dn_fail(DN_ERR_UNSUPPORTED, "dn_dcn_create: channels per deform group must divide 64");
    if (L->cout > 256) return dn_fail(DN_ERR_UNSUPPORTED, "dn_dcn_create: out_channels > 256");
    L->NT = std::max(16, next_pow2(L->cout));
    const int KK = L->kh * L->kw;
    const int K = deform_groups * KK * L->cpg;
    L->k_chunks = (K + kKC - 1) / kKC;
    // B tiles: K index = (g*KK + k)*cpg + c, no-swizzle K-major core matrices.
    const size_t tile = static_cast<size_t>(L->NT) * kKC * 2;
    std::vector<uint8_t> pk(tile * L->k_chunks, 0);
    for (int o = 0; o < L->cout; ++o)
        for (int g = 0; g < deform_groups; ++g)
            for (int k = 0; k < KK; ++k)
                for (int c = 0; c < L->cpg; ++c) {
                    const int kidx = (g * KK + k) * L->cpg + c;
                    const float v = w[((static_cast<size_t>(o) * L->cin + g * L->cpg + c) * KK) + k];
                    const __half h = __float2half(v);
                    const int j = kidx / kKC, kk = kidx % kKC;
                    uint8_t* t = pk.data() + j * tile;
                    const size_t offb = static_cast<size_t>(o >> 3) * 1024 + (kk / 8) * 128 + (o & 7) * 16 + (kk % 8) * 2;
                    std::memcpy(t + offb, &h, 2);
                }
    std::vector<float> b(L->NT, 0.f);
    if (bias)
        for (int o = 0; o < L->cout; ++o) b[o] = __half2float(__float2half(bias[o]));
    DevGuard dg(device);
    cudaError_t e = cudaMalloc(&L->bpack, pk.size());
    if (e == cudaSuccess) e = cudaMalloc(&L->bias, b.size() * 4);
    if (e == cudaSuccess) e = cudaMalloc(&L->err, 4);
    if (e == cudaSuccess) e = cudaMemcpy(L->bpack, pk.data(), pk.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(L->bias, b.data(), b.size() * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(L->err, 0, 4);
    if (e != cudaSuccess) {
        cudaFree(L->bpack);
        cudaFree(L->bias);
        cudaFree(L->err);
        return dn_cuda_fail(e, "dn_dcn_create: upload");
    }
    *out = L.release();
    return DN_OK;
}

int dcn_run_nhwc(dn_dcn* L, const __half* x_nhwc, const __half* off, const __half* msk, const __half* off2,
                 const __half* msk2, int N, int H_in, int W_in, void* output, const DcnFuse* fuse, cudaStream_t s) {
    int Ho = 0, Wo = 0;
    dn_dcn_output_size(L, H_in, W_in, &Ho, &Wo);
    if (Ho <= 0 || Wo <= 0) return dn_fail(DN_ERR_INVALID_ARG, "dn_dcn_forward: output would be empty");
    if (fuse && (N != 1 || L->cout > L->NT)) return dn_fail(DN_ERR_UNSUPPORTED, "dcn fusion epilogue: batch 1 only");
    if ((off2 == nullptr) != (msk2 == nullptr))
        return dn_fail(DN_ERR_INVALID_ARG, "dcn: second offset and mask terms come together");
    DcnParams p{};
    p.xt = x_nhwc;
    p.off = off;
    p.msk = msk;
    p.off2 = off2;
    p.msk2 = msk2;
    p.out = static_cast<__half*>(output);
    p.out_mode = fuse ? kOutFuse : kOutNCHW;
    if (fuse) {
        p.fuse_w = fuse->w;
        p.fuse_acc = fuse->acc;
        p.fuse_out = fuse->out16;
    }
    p.bpack = L->bpack;
    p.bias = L->bias;
    p.N = N;
    p.H = H_in;
    p.W = W_in;
    p.Ho = Ho;
    p.Wo = Wo;
    p.Cin = L->cin;
    p.Cout = L->cout;
    p.kw = L->kw;
    p.KK = L->kh * L->kw;
    p.pad = L->pad;
    p.stride = L->stride;
    p.dil = L->dil;
    p.dg = L->dg;
    p.cpg = L->cpg;
    p.k_chunks = L->k_chunks;
    p.err = L->err;
    p.cout_base = 0;
    return run_conv_nt<true>(p, L->NT, L->device, s);
}

int dcn_nt(const dn_dcn* L) { return L->NT; }

}  // namespace dnb

extern "C" {

int dn_dcn_create(const dn_weights* store, const char* weight_name, const char* bias_name, int pad, int stride,
                  int dilation, int deform_groups, int device, dn_dcn** out) {
    if (!store || !weight_name || !out) return dn_fail(DN_ERR_INVALID_ARG, "dn_dcn_create: null argument");
    *out = nullptr;
    try {
        const HostWeights& hw = *store->hw;
        if (!hw.contains(weight_name)) return dn_fail_str(DN_ERR_NOT_FOUND, std::string("weight not found: ") + weight_name);
        if (bias_name && !hw.contains(bias_name))
            return dn_fail_str(DN_ERR_NOT_FOUND, std::string("weight not found: ") + bias_name);
        const auto& sh = hw.entry(weight_name).shape;
        if (sh.size() != 4)
            return dn_fail_str(DN_ERR_FORMAT, "DeformConv2dLayer: weight must be 4-D, got " + std::to_string(sh.size()) + "-D");
        const auto w = hw.to_f32(weight_name);
        std::vector<float> bv;
        if (bias_name) {
            bv = hw.to_f32(bias_name);
            if (static_cast<int64_t>(bv.size()) != sh[0]) return dn_fail(DN_ERR_FORMAT, "dn_dcn_create: bias size");
        }
        return dnb::dcn_build(w.data(), bias_name ? bv.data() : nullptr, static_cast<int>(sh[0]), static_cast<int>(sh[1]),
                              static_cast<int>(sh[2]), static_cast<int>(sh[3]), pad, stride, dilation, deform_groups,
                              device, out);
    } catch (const std::exception& ex) {
        return dn_fail_str(DN_ERR_FORMAT, ex.what());
    }
}

int dn_dcn_destroy(dn_dcn* L) {
    if (!L) return DN_OK;
    DevGuard dg(L->device);
    cudaFree(L->bpack);
    cudaFree(L->bias);
    cudaFree(L->xt);
    cudaFree(L->err);
    delete L;
    return DN_OK;
}

int dn_dcn_info(const dn_dcn* L, int* out_channels, int* in_channels, int* deform_groups, int* kernel_h,
                int* kernel_w) {
    if (!L) return dn_fail(DN_ERR_INVALID_ARG, "dn_dcn_info: null layer");
    if (out_channels) *out_channels = L->cout;
    if (in_channels) *in_channels = L->cin;
    if (deform_groups) *deform_groups = L->dg;
    if (kernel_h) *kernel_h = L->kh;
    if (kernel_w) *kernel_w = L->kw;
    return DN_OK;
}

int dn_dcn_output_size(const dn_dcn* L, int H_in, int W_in, int* H_out, int* W_out) {
    if (!L || !H_out || !W_out) return dn_fail(DN_ERR_INVALID_ARG, "dn_dcn_output_size: null argument");
    *H_out = (H_in + 2 * L->pad - L->dil * (L->kh - 1) - 1) / L->stride + 1;
    *W_out = (W_in + 2 * L->pad - L->dil * (L->kw - 1) - 1) / L->stride + 1;
    return DN_OK;
}

int dn_dcn_forward(dn_dcn* L, const void* input, const void* offsets, const void* masks, int N, int H_in,
                   int W_in, void* output, void* stream) {
    if (!L || !input || !offsets || !masks || !output)
        return dn_fail(DN_ERR_INVALID_ARG, "dn_dcn_forward: null argument");
    if (N <= 0 || H_in <= 0 || W_in <= 0) return dn_fail(DN_ERR_INVALID_ARG, "dn_dcn_forward: empty input");
    int Ho = 0, Wo = 0;
    dn_dcn_output_size(L, H_in, W_in, &Ho, &Wo);
    if (Ho <= 0 || Wo <= 0) return dn_fail(DN_ERR_INVALID_ARG, "dn_dcn_forward: output would be empty");
    if (static_cast<long long>(N) * H_in * W_in * L->cin > (1LL << 31))
        return dn_fail(DN_ERR_UNSUPPORTED, "dn_dcn_forward: input too large");
    DevGuard dg(L->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t need = static_cast<size_t>(N) * H_in * W_in * L->cin * 2;
    if (need > L->xt_bytes) {
        cudaError_t e = cudaStreamSynchronize(s);  // the old copy may still be read
        if (e == cudaSuccess) {
            cudaFree(L->xt);
            L->xt = nullptr;
            L->xt_bytes = 0;
            e = cudaMalloc(&L->xt, need);
        }
        if (e != cudaSuccess) return dn_cuda_fail(e, "dn_dcn_forward: NHWC buffer");
        L->xt_bytes = need;
    }
    const int HW = H_in * W_in;
    cudaError_t e = launch_pdl(to_nhwc_kernel, dim3((HW + 31) / 32, (L->cin + 31) / 32, N), dim3(32, 8), 0, s,
                               static_cast<const __half*>(input), L->xt, L->cin, HW);
    if (e != cudaSuccess) return dn_cuda_fail(e, "dn_dcn_forward: transpose launch");
    return dnb::dcn_run_nhwc(L, L->xt, static_cast<const __half*>(offsets), static_cast<const __half*>(masks), nullptr,
                             nullptr, N, H_in, W_in, output, nullptr, s);
}

int dn_dcn_sync(dn_dcn* L, void* stream) {
    if (!L) return dn_fail(DN_ERR_INVALID_ARG, "dn_dcn_sync: null layer");
    DevGuard dg(L->device);
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return dn_cuda_fail(e, "dn_dcn_sync");
    uint32_t word = 0;
    e = cudaMemcpy(&word, L->err, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return dn_cuda_fail(e, "dn_dcn_sync: error word");
    if (word) {
        cudaMemset(L->err, 0, 4);
        return dn_fail_str(DN_ERR_DEVICE, "dcn kernel reported device error word " + std::to_string(word));
    }
    return DN_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Conv2dLayer
// ---------------------------------------------------------------------------

struct dn_conv2d {
    int device = 0;
    int cout = 0, cin_g = 0, cin = 0, kh = 0, kw = 0, pad = 1, stride = 1, dil = 1, groups = 1;
    int cb = 0, nblk = 0, NT = 0, slabs = 0, k_chunks = 0;
    uint8_t* bpack = nullptr;  // device: [slabs][k_chunks][NT x 64] packed weights
    float* bias = nullptr;     // device: [slabs * NT]
    __half* xt = nullptr;      // device: NHWC copy of the input (grown on demand)
    size_t xt_bytes = 0;
    uint32_t* err = nullptr;
};

namespace dnb {

int conv2d_build(const float* w, const float* bias, int cout, int cin_g, int kh, int kw, int pad, int stride,
                 int dilation, int groups, int device, dn_conv2d** out) {
    *out = nullptr;
    if (pad < 0 || stride <= 0 || dilation <= 0 || groups <= 0 || cout <= 0 || cin_g <= 0 || kh <= 0 || kw <= 0)
        return dn_fail(DN_ERR_INVALID_ARG, "dn_conv2d_create: bad pad/stride/dilation/groups");
    auto L = std::make_unique<dn_conv2d>();
    L->device = device;
    L->cout = cout;
    L->cin_g = cin_g;
    L->kh = kh;
    L->kw = kw;
    L->pad = pad;
    L->stride = stride;
    L->dil = dilation;
    L->groups = groups;
    if (L->cout % groups != 0) return dn_fail(DN_ERR_INVALID_ARG, "dn_conv2d_create: out_channels % groups != 0");
    L->cin = L->cin_g * groups;
    L->cb = kKC;
    while (L->cin % L->cb != 0) L->cb >>= 1;  // largest power of two dividing Cin and 64
    L->nblk = L->cin / L->cb;
    const int KK = L->kh * L->kw;
    L->k_chunks = (L->cin * KK + kKC - 1) / kKC;
    L->NT = std::min(256, std::max(16, next_pow2(L->cout)));
    L->slabs = (L->cout + L->NT - 1) / L->NT;
    const size_t tile = static_cast<size_t>(L->NT) * kKC * 2;
    const size_t slab_bytes = tile * L->k_chunks;
    std::vector<uint8_t> pk(slab_bytes * L->slabs, 0);
    const int cout_g = L->cout / groups;
    for (int o = 0; o < L->cout; ++o) {
        const int sl = o / L->NT, ol = o % L->NT, grp = o / cout_g;
        for (int cl = 0; cl < L->cin_g; ++cl) {
            const int ci = grp * L->cin_g + cl;
            for (int k = 0; k < KK; ++k) {
                const int kidx = ((ci / L->cb) * KK + k) * L->cb + (ci % L->cb);
                const __half h = __float2half(w[(static_cast<size_t>(o) * L->cin_g + cl) * KK + k]);
                const int j = kidx / kKC, kk = kidx % kKC;
                const size_t offb = static_cast<size_t>(ol >> 3) * 1024 + (kk / 8) * 128 + (ol & 7) * 16 + (kk % 8) * 2;
                std::memcpy(pk.data() + sl * slab_bytes + j * tile + offb, &h, 2);
            }
        }
    }
    std::vector<float> b(static_cast<size_t>(L->slabs) * L->NT, 0.f);
    if (bias)
        for (int o = 0; o < L->cout; ++o) b[o] = __half2float(__float2half(bias[o]));
    DevGuard dg(device);
    cudaError_t e = cudaMalloc(&L->bpack, pk.size());
    if (e == cudaSuccess) e = cudaMalloc(&L->bias, b.size() * 4);
    if (e == cudaSuccess) e = cudaMalloc(&L->err, 4);
    if (e == cudaSuccess) e = cudaMemcpy(L->bpack, pk.data(), pk.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(L->bias, b.data(), b.size() * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(L->err, 0, 4);
    if (e != cudaSuccess) {
        cudaFree(L->bpack);
        cudaFree(L->bias);
        cudaFree(L->err);
        return dn_cuda_fail(e, "dn_conv2d_create: upload");
    }
    *out = L.release();
    return DN_OK;
}

int conv2d_run_nhwc(dn_conv2d* L, const __half* x_nhwc, int N, int H_in, int W_in, void* output, bool out_nhwc,
                    cudaStream_t s) {
    int Ho = 0, Wo = 0;
    dn_conv2d_output_size(L, H_in, W_in, &Ho, &Wo);
    if (Ho <= 0 || Wo <= 0) return dn_fail(DN_ERR_INVALID_ARG, "dn_conv2d_forward: output would be empty");
    DcnParams p{};
    p.xt = x_nhwc;
    p.out = static_cast<__half*>(output);
    p.out_mode = out_nhwc ? kOutNHWC : kOutNCHW;
    p.N = N;
    p.H = H_in;
    p.W = W_in;
    p.Ho = Ho;
    p.Wo = Wo;
    p.Cin = L->cin;
    p.Cout = L->cout;
    p.kw = L->kw;
    p.KK = L->kh * L->kw;
    p.pad = L->pad;
    p.stride = L->stride;
    p.dil = L->dil;
    p.dg = L->nblk;
    p.cpg = L->cb;
    p.k_chunks = L->k_chunks;
    p.err = L->err;
    const size_t slab_bytes = static_cast<size_t>(L->NT) * kKC * 2 * L->k_chunks;
    for (int sl = 0; sl < L->slabs; ++sl) {
        p.bpack = L->bpack + sl * slab_bytes;
        p.bias = L->bias + sl * L->NT;
        p.cout_base = sl * L->NT;
        DN_TRY(run_conv_nt<false>(p, L->NT, L->device, s));
    }
    return DN_OK;
}

int conv2d_to_nhwc(const __half* in, __half* out, int N, int C, int HW, cudaStream_t s) {
    cudaError_t e = launch_pdl(to_nhwc_kernel, dim3((HW + 31) / 32, (C + 31) / 32, N), dim3(32, 8), 0, s, in, out, C, HW);
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "NCHW -> NHWC transpose launch");
}

int conv2d_check(dn_conv2d* L) {
    uint32_t word = 0;
    cudaError_t e = cudaMemcpy(&word, L->err, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return dn_cuda_fail(e, "conv error word");
    if (word) {
        cudaMemset(L->err, 0, 4);
        return dn_fail_str(DN_ERR_DEVICE, "conv kernel reported device error word " + std::to_string(word));
    }
    return DN_OK;
}

int dcn_check(dn_dcn* L) {
    uint32_t word = 0;
    cudaError_t e = cudaMemcpy(&word, L->err, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return dn_cuda_fail(e, "dcn error word");
    if (word) {
        cudaMemset(L->err, 0, 4);
        return dn_fail_str(DN_ERR_DEVICE, "dcn kernel reported device error word " + std::to_string(word));
    }
    return DN_OK;
}

}  // namespace dnb

extern "C" {

int dn_conv2d_create(const dn_weights* store, const char* weight_name, const char* bias_name, int pad, int stride,
                     int dilation, int groups, int device, dn_conv2d** out) {
    if (!store || !weight_name || !out) return dn_fail(DN_ERR_INVALID_ARG, "dn_conv2d_create: null argument");
    *out = nullptr;
    try {
        const HostWeights& hw = *store->hw;
        if (!hw.contains(weight_name)) return dn_fail_str(DN_ERR_NOT_FOUND, std::string("weight not found: ") + weight_name);
        if (bias_name && !hw.contains(bias_name))
            return dn_fail_str(DN_ERR_NOT_FOUND, std::string("weight not found: ") + bias_name);
        const auto& sh = hw.entry(weight_name).shape;
        if (sh.size() != 4)
            return dn_fail_str(DN_ERR_FORMAT, "Conv2dLayer: weight must be 4-D, got " + std::to_string(sh.size()) + "-D");
        const auto w = hw.to_f32(weight_name);
        std::vector<float> bv;
        if (bias_name) {
            bv = hw.to_f32(bias_name);
            if (static_cast<int64_t>(bv.size()) != sh[0]) return dn_fail(DN_ERR_FORMAT, "dn_conv2d_create: bias size");
        }
        return dnb::conv2d_build(w.data(), bias_name ? bv.data() : nullptr, static_cast<int>(sh[0]),
                                 static_cast<int>(sh[1]), static_cast<int>(sh[2]), static_cast<int>(sh[3]), pad, stride,
                                 dilation, groups, device, out);
    } catch (const std::exception& ex) {
        return dn_fail_str(DN_ERR_FORMAT, ex.what());
    }
}

int dn_conv2d_destroy(dn_conv2d* L) {
    if (!L) return DN_OK;
    DevGuard dg(L->device);
    cudaFree(L->bpack);
    cudaFree(L->bias);
    cudaFree(L->xt);
    cudaFree(L->err);
    delete L;
    return DN_OK;
}

int dn_conv2d_info(const dn_conv2d* L, int* out_channels, int* in_channels, int* kernel_h, int* kernel_w,
                   int* groups) {
    if (!L) return dn_fail(DN_ERR_INVALID_ARG, "dn_conv2d_info: null layer");
    if (out_channels) *out_channels = L->cout;
    if (in_channels) *in_channels = L->cin_g;
    if (kernel_h) *kernel_h = L->kh;
    if (kernel_w) *kernel_w = L->kw;
    if (groups) *groups = L->groups;
    return DN_OK;
}

int dn_conv2d_output_size(const dn_conv2d* L, int H_in, int W_in, int* H_out, int* W_out) {
    if (!L || !H_out || !W_out) return dn_fail(DN_ERR_INVALID_ARG, "dn_conv2d_output_size: null argument");
    *H_out = (H_in + 2 * L->pad - L->dil * (L->kh - 1) - 1) / L->stride + 1;
    *W_out = (W_in + 2 * L->pad - L->dil * (L->kw - 1) - 1) / L->stride + 1;
    return DN_OK;
}

int dn_conv2d_forward(dn_conv2d* L, const void* input, int N, int C, int H_in, int W_in, void* output, void* stream) {
    if (!L || !input || !output) return dn_fail(DN_ERR_INVALID_ARG, "dn_conv2d_forward: null argument");
    if (N <= 0 || H_in <= 0 || W_in <= 0) return dn_fail(DN_ERR_INVALID_ARG, "dn_conv2d_forward: empty input");
    if (C != L->cin)
        return dn_fail_str(DN_ERR_INVALID_ARG, "dn_conv2d_forward: input has " + std::to_string(C) +
                                                   " channels, the layer expects " + std::to_string(L->cin));
    int Ho = 0, Wo = 0;
    dn_conv2d_output_size(L, H_in, W_in, &Ho, &Wo);
    if (Ho <= 0 || Wo <= 0) return dn_fail(DN_ERR_INVALID_ARG, "dn_conv2d_forward: output would be empty");
    if (static_cast<long long>(N) * H_in * W_in * L->cin > (1LL << 31) ||
        static_cast<long long>(N) * Ho * Wo > (1LL << 31))
        return dn_fail(DN_ERR_UNSUPPORTED, "dn_conv2d_forward: input too large");
    DevGuard dg(L->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t need = static_cast<size_t>(N) * H_in * W_in * L->cin * 2;
    if (need > L->xt_bytes) {
        cudaError_t e = cudaStreamSynchronize(s);  // the old copy may still be read
        if (e == cudaSuccess) {
            cudaFree(L->xt);
            L->xt = nullptr;
            L->xt_bytes = 0;
            e = cudaMalloc(&L->xt, need);
        }
        if (e != cudaSuccess) return dn_cuda_fail(e, "dn_conv2d_forward: NHWC buffer");
        L->xt_bytes = need;
    }
    DN_TRY(dnb::conv2d_to_nhwc(static_cast<const __half*>(input), L->xt, N, L->cin, H_in * W_in, s));
    return dnb::conv2d_run_nhwc(L, L->xt, N, H_in, W_in, output, false, s);
}

int dn_conv2d_sync(dn_conv2d* L, void* stream) {
    if (!L) return dn_fail(DN_ERR_INVALID_ARG, "dn_conv2d_sync: null layer");
    DevGuard dg(L->device);
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return dn_cuda_fail(e, "dn_conv2d_sync");
    uint32_t word = 0;
    e = cudaMemcpy(&word, L->err, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return dn_cuda_fail(e, "dn_conv2d_sync: error word");
    if (word) {
        cudaMemset(L->err, 0, 4);
        return dn_fail_str(DN_ERR_DEVICE, "conv kernel reported device error word " + std::to_string(word));
    }
    return DN_OK;
}

}  // extern "C"
