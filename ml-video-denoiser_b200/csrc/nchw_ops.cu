// NCHW FP16 kernel launchers behind include/denoiser_b200_ops.h.
//
// These are the reference's denoiser::kernels::launch_* operations
// (src/kernels/model_kernels.cu:15-115, src/kernels/nafnet_kernels.cu:16-406,
// src/kernels/concat.cuh:19-41) with the same element-wise arithmetic (FP32
// math on FP16 loads, one round-to-nearest FP16 store), re-laid for B200:
//   * every kernel is HBM-bound, so each moves 16-byte vectors (8 halves)
//     whenever sizes and pointers allow it and falls back to scalar accesses
//     otherwise; grids are sized to a multiple of the SM count and stride;
//   * copies (pad, crop, extract, prefix, concat) run one warp per row so a
//     row is read and written with contiguous vectors;
//   * LayerNorm stages a 64-pixel x C tile in shared memory, so the input is
//     read from HBM once (the reference reads it three times);
//   * the global average pool splits every plane across thread blocks (the
//     reference runs one thread per plane) and adds the split sums in a fixed
//     order, so the mean is deterministic.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <mutex>
#include <string>

#include "denoiser_b200.h"
#include "denoiser_b200_ops.h"
#include "status.h"

namespace dnb {
namespace {

constexpr int kThreads = 256;

int sm_count() {
    static std::atomic<int> cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    int v = cache[dev].load(std::memory_order_relaxed);
    if (v == 0) {
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        cache[dev].store(v, std::memory_order_relaxed);
    }
    return v;
}

// Blocks for `work` items of `per_block` each, capped at 16 blocks per SM
// (every kernel strides over its items).
unsigned grid_for(int64_t work, int64_t per_block) {
    const int64_t want = (work + per_block - 1) / per_block;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
    return static_cast<unsigned>(std::max<int64_t>(1, std::min(want, cap)));
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
bool al4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3) == 0; }

cudaStream_t to_stream(void* s) { return static_cast<cudaStream_t>(s); }

int launched(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return dn_cuda_fail(e, what);
    return DN_OK;
}

__device__ __forceinline__ void load8(const __half* p, float f[8]) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    const uint32_t q[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        __half2 h;
        memcpy(&h, &q[i], 4);
        const float2 t = __half22float2(h);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

__device__ __forceinline__ void store8(__half* p, const float f[8]) {
    uint32_t q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
        memcpy(&q[i], &h, 4);
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(q[0], q[1], q[2], q[3]);
}

__device__ __forceinline__ float read_param(const void* p, bool fp32, int i) {
    return fp32 ? static_cast<const float*>(p)[i] : __half2float(static_cast<const __half*>(p)[i]);
}

// ---------------------------------------------------------------------------
// Flat element-wise ops: add, mul_scalar, subtract_clamp
// ---------------------------------------------------------------------------

enum FlatOp { kAdd = 0, kMulScalar = 1, kSubClamp = 2 };

template <int OP>
__device__ __forceinline__ float flat_op(float a, float b, float s) {
    if constexpr (OP == kAdd) return a + b;
    if constexpr (OP == kMulScalar) return a * s;
    const float v = a - b;
    return v < 0.f ? 0.f : (v > 1.f ? 1.f : v);
}

template <int OP, bool VEC>
__global__ void __launch_bounds__(kThreads) flat_kernel(const __half* __restrict__ a, const __half* __restrict__ b,
                                                        float s, __half* __restrict__ out, int64_t n) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    int64_t tail = 0;
    if constexpr (VEC) {
        const int64_t nv = n >> 3;
        for (int64_t v = t; v < nv; v += stride) {
            float fa[8], fb[8], o[8];
            load8(a + v * 8, fa);
            if constexpr (OP != kMulScalar) load8(b + v * 8, fb);
#pragma unroll
            for (int k = 0; k < 8; ++k) o[k] = flat_op<OP>(fa[k], OP != kMulScalar ? fb[k] : 0.f, s);
            store8(out + v * 8, o);
        }
        tail = nv * 8;
    }
    for (int64_t i = tail + t; i < n; i += stride) {
        const float fb = OP != kMulScalar ? __half2float(b[i]) : 0.f;
        out[i] = __float2half(flat_op<OP>(__half2float(a[i]), fb, s));
    }
}

template <int OP>
int run_flat(const void* a, const void* b, float s, void* out, int64_t n, void* stream, const char* name) {
    if (n < 0) return dn_fail_str(DN_ERR_INVALID_ARG, std::string(name) + ": negative element count");
    if (n == 0) return DN_OK;
    if (!a || !out || (OP != kMulScalar && !b)) return dn_fail_str(DN_ERR_INVALID_ARG, std::string(name) + ": null pointer");
    const auto* ha = static_cast<const __half*>(a);
    const auto* hb = static_cast<const __half*>(b);
    auto* ho = static_cast<__half*>(out);
    const bool vec = al16(a) && al16(out) && (OP == kMulScalar || al16(b));
    if (vec)
        flat_kernel<OP, true><<<grid_for(n, kThreads * 8), kThreads, 0, to_stream(stream)>>>(ha, hb, s, ho, n);
    else
        flat_kernel<OP, false><<<grid_for(n, kThreads), kThreads, 0, to_stream(stream)>>>(ha, hb, s, ho, n);
    return launched(name);
}

// ---------------------------------------------------------------------------
// Per-channel ops: mul_channelwise (scale[n*C + c]) and scaled_add (scale[c])
// ---------------------------------------------------------------------------

template <bool SCALED_ADD, bool VEC>
__global__ void __launch_bounds__(kThreads)
    chan_kernel(const __half* __restrict__ x, const __half* __restrict__ r, const void* __restrict__ scale,
                bool scale_fp32, __half* __restrict__ out, int C, int64_t HW, int64_t total) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if constexpr (VEC) {
        // HW % 8 == 0: a vector never crosses a plane
        for (int64_t v = t; v < (total >> 3); v += stride) {
            const int64_t i = v * 8;
            const int64_t plane = i / HW;
            float s;
            if constexpr (SCALED_ADD)
                s = read_param(scale, scale_fp32, static_cast<int>(plane % C));
            else
                s = __half2float(static_cast<const __half*>(scale)[plane]);
            float fx[8], o[8];
            load8(x + i, fx);
            if constexpr (SCALED_ADD) {
                float fr[8];
                load8(r + i, fr);
#pragma unroll
                for (int k = 0; k < 8; ++k) o[k] = fx[k] + fr[k] * s;
            } else {
#pragma unroll
                for (int k = 0; k < 8; ++k) o[k] = fx[k] * s;
            }
            store8(out + i, o);
        }
    } else {
        for (int64_t i = t; i < total; i += stride) {
            const int64_t plane = i / HW;
            if constexpr (SCALED_ADD) {
                const float s = read_param(scale, scale_fp32, static_cast<int>(plane % C));
                out[i] = __float2half(__half2float(x[i]) + __half2float(r[i]) * s);
            } else {
                const float s = __half2float(static_cast<const __half*>(scale)[plane]);
                out[i] = __float2half(__half2float(x[i]) * s);
            }
        }
    }
}

template <bool SCALED_ADD>
int run_chan(const void* x, const void* r, const void* scale, bool s32, void* out, int N, int C, int H, int W,
             void* stream, const char* name) {
    if (N < 0 || C < 0 || H < 0 || W < 0) return dn_fail_str(DN_ERR_INVALID_ARG, std::string(name) + ": negative size");
    const int64_t HW = static_cast<int64_t>(H) * W;
    const int64_t total = static_cast<int64_t>(N) * C * HW;
    if (total == 0) return DN_OK;
    if (!x || !scale || !out || (SCALED_ADD && !r))
        return dn_fail_str(DN_ERR_INVALID_ARG, std::string(name) + ": null pointer");
    const auto* hx = static_cast<const __half*>(x);
    const auto* hr = static_cast<const __half*>(r);
    auto* ho = static_cast<__half*>(out);
    const bool vec = HW % 8 == 0 && al16(x) && al16(out) && (!SCALED_ADD || al16(r));
    if (vec)
        chan_kernel<SCALED_ADD, true><<<grid_for(total, kThreads * 8), kThreads, 0, to_stream(stream)>>>(
            hx, hr, scale, s32, ho, C, HW, total);
    else
        chan_kernel<SCALED_ADD, false><<<grid_for(total, kThreads), kThreads, 0, to_stream(stream)>>>(
            hx, hr, scale, s32, ho, C, HW, total);
    return launched(name);
}

// ---------------------------------------------------------------------------
// SimpleGate: out[n, c] = in[n, c] * in[n, C + c]
// ---------------------------------------------------------------------------

template <bool VEC>
__global__ void __launch_bounds__(kThreads)
    gate_kernel(const __half* __restrict__ in, __half* __restrict__ out, int64_t CHW, int64_t total) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if constexpr (VEC) {
        for (int64_t v = t; v < (total >> 3); v += stride) {
            const int64_t i = v * 8;
            const int64_t n = i / CHW;
            const int64_t src = i + n * CHW;  // n * 2CHW + (i - n * CHW)
            float a[8], b[8], o[8];
            load8(in + src, a);
            load8(in + src + CHW, b);
#pragma unroll
            for (int k = 0; k < 8; ++k) o[k] = a[k] * b[k];
            store8(out + i, o);
        }
    } else {
        for (int64_t i = t; i < total; i += stride) {
            const int64_t src = i + (i / CHW) * CHW;
            out[i] = __float2half(__half2float(in[src]) * __half2float(in[src + CHW]));
        }
    }
}

// ---------------------------------------------------------------------------
// LayerNorm over channels of NCHW: one CTA per (image, TP-pixel tile)
// ---------------------------------------------------------------------------

template <int TP>
__global__ void __launch_bounds__(kThreads)
    ln_kernel(const __half* __restrict__ in, const void* __restrict__ w, const void* __restrict__ b, bool p32,
              __half* __restrict__ out, int C, int64_t HW, int64_t tiles_per_img) {
    extern __shared__ __align__(16) __half s_tile[];  // [C][TP]
    __shared__ float s_red[kThreads];
    __shared__ float s_mean[TP], s_rstd[TP];
    constexpr int KP = kThreads / TP;
    const int64_t tile = blockIdx.x;
    const int64_t n = tile / tiles_per_img;
    const int64_t p0 = (tile - n * tiles_per_img) * TP;
    const int q = threadIdx.x % TP, k = threadIdx.x / TP;
    const bool valid = p0 + q < HW;
    const __half* src = in + n * C * HW + p0 + q;
    __half* dst = out + n * C * HW + p0 + q;

    for (int c = k; c < C; c += KP) s_tile[c * TP + q] = valid ? src[c * HW] : __float2half(0.f);
    __syncthreads();
    float sum = 0.f;
    for (int c = k; c < C; c += KP) sum += __half2float(s_tile[c * TP + q]);
    s_red[threadIdx.x] = sum;
    __syncthreads();
    if (k == 0) {
        float m = 0.f;
#pragma unroll
        for (int j = 0; j < KP; ++j) m += s_red[j * TP + q];
        s_mean[q] = m / static_cast<float>(C);
    }
    __syncthreads();
    const float mean = s_mean[q];
    float var = 0.f;
    for (int c = k; c < C; c += KP) {
        const float d = __half2float(s_tile[c * TP + q]) - mean;
        var += d * d;
    }
    s_red[threadIdx.x] = var;
    __syncthreads();
    if (k == 0) {
        float v = 0.f;
#pragma unroll
        for (int j = 0; j < KP; ++j) v += s_red[j * TP + q];
        s_rstd[q] = rsqrtf(v / static_cast<float>(C) + 1e-6f);
    }
    __syncthreads();
    if (!valid) return;
    const float rstd = s_rstd[q];
    for (int c = k; c < C; c += KP) {
        const float norm = (__half2float(s_tile[c * TP + q]) - mean) * rstd;
        dst[c * HW] = __float2half(norm * read_param(w, p32, c) + read_param(b, p32, c));
    }
}

// ---------------------------------------------------------------------------
// Global average pool: split sums, then a fixed-order reduction per plane
// ---------------------------------------------------------------------------

constexpr int64_t kPoolChunk = 16384;  // elements per split (target)
constexpr int kPoolMaxSplits = 128;

template <bool VEC>
__global__ void __launch_bounds__(kThreads)
    pool_split_kernel(const __half* __restrict__ in, float* __restrict__ partials, int64_t HW, int splits,
                      int64_t chunk) {
    __shared__ float s_warp[kThreads / 32];
    const int64_t plane = blockIdx.x / splits;
    const int split = static_cast<int>(blockIdx.x - plane * splits);
    const int64_t b0 = split * chunk;
    const int64_t e0 = std::min<int64_t>(HW, b0 + chunk);
    const __half* src = in + plane * HW;
    float acc = 0.f;
    if constexpr (VEC) {
        // HW % 8 == 0 and chunk % 8 == 0: [b0, e0) is whole vectors
        for (int64_t e = b0 + threadIdx.x * 8; e < e0; e += kThreads * 8) {
            float f[8];
            load8(src + e, f);
#pragma unroll
            for (int k = 0; k < 8; ++k) acc += f[k];
        }
    } else {
        for (int64_t e = b0 + threadIdx.x; e < e0; e += kThreads) acc += __half2float(src[e]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) s_warp[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < kThreads / 32; ++j) s += s_warp[j];
        partials[blockIdx.x] = s;
    }
}

__global__ void __launch_bounds__(kThreads)
    pool_final_kernel(const float* __restrict__ partials, __half* __restrict__ out, int64_t planes, int splits,
                      int64_t HW) {
    const int64_t plane = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (plane >= planes) return;
    const float* p = partials + plane * splits;
    float s = 0.f;
    for (int j = 0; j < splits; ++j) s += p[j];
    out[plane] = __float2half(s / static_cast<float>(HW));
}

struct PoolPlan {
    int64_t planes, HW, chunk;
    int splits;
    bool vec;
};

PoolPlan pool_plan(const void* input, int N, int C, int H, int W) {
    PoolPlan p{};
    p.planes = static_cast<int64_t>(N) * C;
    p.HW = static_cast<int64_t>(H) * W;
    p.splits = static_cast<int>(std::clamp<int64_t>((p.HW + kPoolChunk - 1) / kPoolChunk, 1, kPoolMaxSplits));
    p.vec = p.HW % 8 == 0 && al16(input);
    p.chunk = (p.HW + p.splits - 1) / p.splits;
    if (p.vec) p.chunk = (p.chunk + 7) / 8 * 8;
    return p;
}

int pool_check(const void* input, const void* output, int N, int C, int H, int W, const char* name) {
    if (N < 0 || C < 0 || H < 0 || W < 0) return dn_fail_str(DN_ERR_INVALID_ARG, std::string(name) + ": negative size");
    if (static_cast<int64_t>(N) * C > 0 && (!input || !output))
        return dn_fail_str(DN_ERR_INVALID_ARG, std::string(name) + ": null pointer");
    if (static_cast<int64_t>(N) * C > 0 && static_cast<int64_t>(H) * W == 0)
        return dn_fail_str(DN_ERR_INVALID_ARG, std::string(name) + ": mean over an empty plane");
    return DN_OK;
}

int pool_launch(const PoolPlan& pp, const void* input, void* output, float* partials, cudaStream_t s, const char* name) {
    const auto* hin = static_cast<const __half*>(input);
    const int64_t blocks = pp.planes * pp.splits;
    if (blocks > 0x7fffffffLL) return dn_fail_str(DN_ERR_UNSUPPORTED, std::string(name) + ": too many planes");
    if (pp.vec)
        pool_split_kernel<true><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(hin, partials, pp.HW, pp.splits,
                                                                                  pp.chunk);
    else
        pool_split_kernel<false><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(hin, partials, pp.HW, pp.splits,
                                                                                   pp.chunk);
    DN_TRY(launched(name));
    pool_final_kernel<<<static_cast<unsigned>((pp.planes + kThreads - 1) / kThreads), kThreads, 0, s>>>(
        partials, static_cast<__half*>(output), pp.planes, pp.splits, pp.HW);
    return launched(name);
}

// ---------------------------------------------------------------------------
// PixelShuffle(2): out[n, co, ho, wo] = in[n, 4co + 2(ho&1) + (wo&1), ho>>1, wo>>1]
// ---------------------------------------------------------------------------

template <bool PAIR>
__global__ void __launch_bounds__(kThreads)
    shuffle_kernel(const __half* __restrict__ in, __half* __restrict__ out, int Cout, int H, int W, int64_t total) {
    // one item = the output pair (ho, 2wi), (ho, 2wi+1)
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int wi = static_cast<int>(i % W);
        int64_t r = i / W;
        const int ho = static_cast<int>(r % (2 * H));
        r /= 2 * H;  // n * Cout + co
        const int64_t n = r / Cout, co = r - n * Cout;
        const int64_t cin0 = co * 4 + (ho & 1) * 2;
        const int64_t src = ((n * Cout * 4 + cin0) * H + (ho >> 1)) * W + wi;
        const __half a = in[src];
        const __half b = in[src + static_cast<int64_t>(H) * W];
        __half* dst = out + (r * 2 * H + ho) * 2 * W + 2 * wi;
        if constexpr (PAIR) {
            *reinterpret_cast<__half2*>(dst) = __halves2half2(a, b);
        } else {
            dst[0] = a;
            dst[1] = b;
        }
    }
}

// ---------------------------------------------------------------------------
// Bilinear warp with pixel offsets, border clamp: one thread per pixel, all C
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(kThreads)
    warp_kernel(const __half* __restrict__ feat, const __half* __restrict__ off, __half* __restrict__ out, int C,
                int H, int W, int64_t total) {
    const int64_t HW = static_cast<int64_t>(H) * W;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int64_t n = i / HW, p = i - n * HW;
        const int h = static_cast<int>(p / W), w = static_cast<int>(p % W);
        const float dx = __half2float(off[n * 2 * HW + p]);
        const float dy = __half2float(off[(n * 2 + 1) * HW + p]);
        const float x = static_cast<float>(w) + dx;
        const float y = static_cast<float>(h) + dy;
        const float fx0 = floorf(x), fy0 = floorf(y);
        const int x0 = static_cast<int>(fx0), y0 = static_cast<int>(fy0);
        const float wx = x - fx0, wy = y - fy0;
        const int xa = min(max(x0, 0), W - 1), xb = min(max(x0 + 1, 0), W - 1);
        const int ya = min(max(y0, 0), H - 1), yb = min(max(y0 + 1, 0), H - 1);
        const int64_t o00 = static_cast<int64_t>(ya) * W + xa, o01 = static_cast<int64_t>(ya) * W + xb;
        const int64_t o10 = static_cast<int64_t>(yb) * W + xa, o11 = static_cast<int64_t>(yb) * W + xb;
        const __half* f = feat + n * C * HW;
        __half* o = out + n * C * HW + p;
        for (int c = 0; c < C; ++c, f += HW) {
            const float v00 = __half2float(f[o00]), v01 = __half2float(f[o01]);
            const float v10 = __half2float(f[o10]), v11 = __half2float(f[o11]);
            const float val = v00 * (1.f - wy) * (1.f - wx) + v01 * (1.f - wy) * wx + v10 * wy * (1.f - wx) +
                              v11 * wy * wx;
            o[c * HW] = __float2half(val);
        }
    }
}

// ---------------------------------------------------------------------------
// Bilinear upsampling by an integer factor (UpsampleLayer's kernel,
// src/layers/upsample.cu:10-45): source coordinate (o + 0.5) / s - 0.5, the
// low corner clamped to >= 0 but the weight taken from the unclamped
// coordinate, so the first output row/column extrapolates slightly (as the
// reference does); the high corner is clamped to the last row/column.
// One thread = one output element; consecutive threads write consecutive
// columns.
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(kThreads)
    upsample_kernel(const __half* __restrict__ in, __half* __restrict__ out, int H, int W, int Ho, int Wo,
                    float scale, int64_t total) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int wo = static_cast<int>(i % Wo);
        const int64_t r = i / Wo;
        const int ho = static_cast<int>(r % Ho);
        const int64_t plane = r / Ho;
        const float hf = (static_cast<float>(ho) + 0.5f) / scale - 0.5f;
        const float wf = (static_cast<float>(wo) + 0.5f) / scale - 0.5f;
        const int h0 = max(0, static_cast<int>(floorf(hf)));
        const int w0 = max(0, static_cast<int>(floorf(wf)));
        const int h1 = min(h0 + 1, H - 1);
        const int w1 = min(w0 + 1, W - 1);
        const float dh = hf - static_cast<float>(h0);
        const float dw = wf - static_cast<float>(w0);
        const __half* src = in + plane * H * W;
        const float v00 = __half2float(src[static_cast<int64_t>(h0) * W + w0]);
        const float v01 = __half2float(src[static_cast<int64_t>(h0) * W + w1]);
        const float v10 = __half2float(src[static_cast<int64_t>(h1) * W + w0]);
        const float v11 = __half2float(src[static_cast<int64_t>(h1) * W + w1]);
        const float val = v00 * (1.f - dh) * (1.f - dw) + v01 * (1.f - dh) * dw + v10 * dh * (1.f - dw) +
                          v11 * dh * dw;
        out[i] = __float2half(val);
    }
}

// ---------------------------------------------------------------------------
// Row copies (pad / crop / extract / prefix / concat): one warp per row
// ---------------------------------------------------------------------------

enum RowMode { kRowCrop = 0, kRowReflect = 1, kRowBlocks = 2, kRowConcat = 3 };

struct RowMap {
    int mode;
    const __half* a;
    const __half* b;
    int64_t rows;      // output rows
    int64_t len;       // elements copied straight from the source row
    int64_t out_len;   // elements per output row (len + reflected tail)
    // crop / reflect: rows are (plane, h) of H_out; source row stride W_in
    int64_t H_out, H_in, W_in;
    // blocks: row r reads a + r * a_stride (+ a_off)
    int64_t a_stride, a_off;
    // concat: rows are (n, c) planes of length HW over C1 + C2 channels
    int64_t C1, C2;
};

__device__ __forceinline__ const __half* row_src(const RowMap& m, int64_t r) {
    switch (m.mode) {
        case kRowCrop:
        case kRowReflect: {
            const int64_t plane = r / m.H_out, h = r - plane * m.H_out;
            const int64_t hs = h < m.H_in ? h : 2 * (m.H_in - 1) - h;
            return m.a + (plane * m.H_in + hs) * m.W_in;
        }
        case kRowBlocks:
            return m.a + m.a_off + r * m.a_stride;
        default: {
            const int64_t C = m.C1 + m.C2;
            const int64_t n = r / C, c = r - n * C;
            return c < m.C1 ? m.a + (n * m.C1 + c) * m.len : m.b + (n * m.C2 + c - m.C1) * m.len;
        }
    }
}

template <bool VEC>
__global__ void __launch_bounds__(kThreads) rows_kernel(const __grid_constant__ RowMap m, __half* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < m.rows; r += nwarps) {
        const __half* s = row_src(m, r);
        __half* d = out + r * m.out_len;
        if constexpr (VEC) {
            for (int64_t j = lane * 8; j < m.len; j += 256)
                *reinterpret_cast<uint4*>(d + j) = __ldg(reinterpret_cast<const uint4*>(s + j));
        } else {
            for (int64_t j = lane; j < m.len; j += 32) d[j] = s[j];
        }
        for (int64_t j = m.len + lane; j < m.out_len; j += 32) d[j] = s[2 * (m.W_in - 1) - j];
    }
}

// `vec_ok`: every source and destination row start is 16-byte aligned and
// the straight copy is whole vectors.
int run_rows(const RowMap& m, void* out, bool vec_ok, void* stream, const char* name) {
    if (m.rows == 0 || m.out_len == 0) return DN_OK;
    const unsigned grid = grid_for(m.rows, kThreads / 32);
    if (vec_ok)
        rows_kernel<true><<<grid, kThreads, 0, to_stream(stream)>>>(m, static_cast<__half*>(out));
    else
        rows_kernel<false><<<grid, kThreads, 0, to_stream(stream)>>>(m, static_cast<__half*>(out));
    return launched(name);
}

// ---------------------------------------------------------------------------
// Average pool on a static scratch (dn_launch_global_avg_pool_noalloc)
// ---------------------------------------------------------------------------

// Split sums of the no-alloc pool: one array per device, part of this
// library's device code, so it exists once the code is loaded on a device.
constexpr int64_t kNoAllocPoolFloats = 262144;  // 1 MiB
static __device__ __align__(256) float g_pool_scratch[kNoAllocPoolFloats];

std::mutex g_pool_scratch_mu;
float* g_pool_scratch_ptr[64];  // device address of g_pool_scratch, per device ordinal

// Device address of g_pool_scratch on the calling thread's current device,
// looked up (cudaGetSymbolAddress) by the first call on that device. The
// cached address lives as long as the device's primary context: after a
// cudaDeviceReset the module is loaded again and the address may change, so
// a process that resets a device must not call the no-alloc pool on it again.
int pool_scratch(float** out, const char* name) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return dn_cuda_fail(e, name);
    if (dev < 0 || dev >= 64) return dn_fail_str(DN_ERR_UNSUPPORTED, std::string(name) + ": device ordinal >= 64");
    std::lock_guard<std::mutex> lock(g_pool_scratch_mu);
    if (!g_pool_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_pool_scratch);
        if (e != cudaSuccess) return dn_cuda_fail(e, "dn_launch_global_avg_pool_noalloc: cudaGetSymbolAddress");
        g_pool_scratch_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_pool_scratch_ptr[dev];
    return DN_OK;
}

bool any_negative(std::initializer_list<int> v) {
    for (int x : v)
        if (x < 0) return true;
    return false;
}

}  // namespace
}  // namespace dnb

using namespace dnb;

extern "C" {

int dn_launch_reflect_pad(const void* input, void* output, int N, int C, int H_in, int W_in, int H_out, int W_out,
                          void* stream) {
    const char* name = "dn_launch_reflect_pad";
    if (any_negative({N, C, H_in, W_in, H_out, W_out}))
        return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_reflect_pad: negative size");
    const int64_t total = static_cast<int64_t>(N) * C * H_out * W_out;
    if (total == 0) return DN_OK;
    if (H_out < H_in || W_out < W_in || H_out - H_in > H_in - 1 || W_out - W_in > W_in - 1)
        return dn_fail(DN_ERR_INVALID_ARG,
                       "dn_launch_reflect_pad: need H_in <= H_out <= 2*H_in-1 and W_in <= W_out <= 2*W_in-1");
    if (!input || !output) return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_reflect_pad: null pointer");
    RowMap m{};
    m.mode = kRowReflect;
    m.a = static_cast<const __half*>(input);
    m.rows = static_cast<int64_t>(N) * C * H_out;
    m.len = W_in;
    m.out_len = W_out;
    m.H_out = H_out;
    m.H_in = H_in;
    m.W_in = W_in;
    const bool vec = al16(input) && al16(output) && W_in % 8 == 0 && W_out % 8 == 0;
    return run_rows(m, output, vec, stream, name);
}

int dn_launch_crop(const void* input, void* output, int N, int C, int H_in, int W_in, int H_out, int W_out,
                   void* stream) {
    if (any_negative({N, C, H_in, W_in, H_out, W_out}))
        return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_crop: negative size");
    if (H_out > H_in || W_out > W_in)
        return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_crop: output larger than input");
    const int64_t total = static_cast<int64_t>(N) * C * H_out * W_out;
    if (total == 0) return DN_OK;
    if (!input || !output) return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_crop: null pointer");
    RowMap m{};
    m.mode = kRowCrop;
    m.a = static_cast<const __half*>(input);
    m.rows = static_cast<int64_t>(N) * C * H_out;
    m.len = W_out;
    m.out_len = W_out;
    m.H_out = H_out;
    m.H_in = H_in;
    m.W_in = W_in;
    const bool vec = al16(input) && al16(output) && W_in % 8 == 0 && W_out % 8 == 0;
    return run_rows(m, output, vec, stream, "dn_launch_crop");
}

int dn_launch_subtract_clamp(const void* a, const void* b, void* out, int64_t n, void* stream) {
    return run_flat<kSubClamp>(a, b, 0.f, out, n, stream, "dn_launch_subtract_clamp");
}

int dn_launch_concat_channels(const void* a, const void* b, void* output, int N, int C1, int C2, int H, int W,
                              void* stream) {
    if (any_negative({N, C1, C2, H, W})) return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_concat_channels: negative size");
    const int64_t HW = static_cast<int64_t>(H) * W;
    if (static_cast<int64_t>(N) * (C1 + C2) * HW == 0) return DN_OK;
    if (!output || (C1 > 0 && !a) || (C2 > 0 && !b))
        return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_concat_channels: null pointer");
    RowMap m{};
    m.mode = kRowConcat;
    m.a = static_cast<const __half*>(a);
    m.b = static_cast<const __half*>(b);
    m.rows = static_cast<int64_t>(N) * (C1 + C2);
    m.len = HW;
    m.out_len = HW;
    m.C1 = C1;
    m.C2 = C2;
    const bool vec = (C1 == 0 || al16(a)) && (C2 == 0 || al16(b)) && al16(output) && HW % 8 == 0;
    return run_rows(m, output, vec, stream, "dn_launch_concat_channels");
}

int dn_launch_extract_frame(const void* clip, void* frame, int N, int T, int C, int H, int W, int frame_idx,
                            void* stream) {
    if (any_negative({N, T, C, H, W})) return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_extract_frame: negative size");
    const int64_t CHW = static_cast<int64_t>(C) * H * W;
    if (static_cast<int64_t>(N) * CHW == 0) return DN_OK;
    if (frame_idx < 0 || frame_idx >= T)
        return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_extract_frame: frame_idx outside [0, T)");
    if (!clip || !frame) return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_extract_frame: null pointer");
    RowMap m{};
    m.mode = kRowBlocks;
    m.a = static_cast<const __half*>(clip);
    m.rows = N;
    m.len = CHW;
    m.out_len = CHW;
    m.a_stride = static_cast<int64_t>(T) * CHW;
    m.a_off = static_cast<int64_t>(frame_idx) * CHW;
    const bool vec = al16(clip) && al16(frame) && CHW % 8 == 0;
    return run_rows(m, frame, vec, stream, "dn_launch_extract_frame");
}

int dn_launch_select_prefix_channels(const void* input, void* output, int N, int C_in, int C_out, int H, int W,
                                     void* stream) {
    if (any_negative({N, C_in, C_out, H, W}))
        return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_select_prefix_channels: negative size");
    if (C_out > C_in) return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_select_prefix_channels: C_out > C_in");
    const int64_t HW = static_cast<int64_t>(H) * W;
    if (static_cast<int64_t>(N) * C_out * HW == 0) return DN_OK;
    if (!input || !output) return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_select_prefix_channels: null pointer");
    RowMap m{};
    m.mode = kRowBlocks;
    m.a = static_cast<const __half*>(input);
    m.rows = N;
    m.len = static_cast<int64_t>(C_out) * HW;
    m.out_len = m.len;
    m.a_stride = static_cast<int64_t>(C_in) * HW;
    const bool vec = al16(input) && al16(output) && HW % 8 == 0;
    return run_rows(m, output, vec, stream, "dn_launch_select_prefix_channels");
}

int dn_launch_layer_norm_affine(const void* input, const void* weight, const void* bias, int params_fp32,
                                void* output, int N, int C, int H, int W, void* stream) {
    if (any_negative({N, C, H, W})) return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_layer_norm_affine: negative size");
    const int64_t HW = static_cast<int64_t>(H) * W;
    if (static_cast<int64_t>(N) * C * HW == 0) return DN_OK;
    if (C > 2048) return dn_fail(DN_ERR_UNSUPPORTED, "dn_launch_layer_norm_affine: C > 2048");
    if (!input || !weight || !bias || !output)
        return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_layer_norm_affine: null pointer");
    const bool p32 = params_fp32 != 0;
    const auto* hin = static_cast<const __half*>(input);
    auto* hout = static_cast<__half*>(output);
    cudaStream_t s = to_stream(stream);
    if (C <= 1024) {
        constexpr int TP = 64;
        static bool configured = false;
        if (!configured) {
            const cudaError_t e = cudaFuncSetAttribute(ln_kernel<TP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       1024 * TP * 2);
            if (e != cudaSuccess) return dn_cuda_fail(e, "dn_launch_layer_norm_affine: smem attribute");
            configured = true;
        }
        const int64_t tiles = (HW + TP - 1) / TP;
        ln_kernel<TP><<<static_cast<unsigned>(N * tiles), kThreads, static_cast<size_t>(C) * TP * 2, s>>>(
            hin, weight, bias, p32, hout, C, HW, tiles);
    } else {
        constexpr int TP = 32;
        static bool configured = false;
        if (!configured) {
            const cudaError_t e = cudaFuncSetAttribute(ln_kernel<TP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       2048 * TP * 2);
            if (e != cudaSuccess) return dn_cuda_fail(e, "dn_launch_layer_norm_affine: smem attribute");
            configured = true;
        }
        const int64_t tiles = (HW + TP - 1) / TP;
        ln_kernel<TP><<<static_cast<unsigned>(N * tiles), kThreads, static_cast<size_t>(C) * TP * 2, s>>>(
            hin, weight, bias, p32, hout, C, HW, tiles);
    }
    return launched("dn_launch_layer_norm_affine");
}

int dn_launch_simple_gate(const void* input, void* output, int N, int C, int H, int W, void* stream) {
    if (any_negative({N, C, H, W})) return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_simple_gate: negative size");
    const int64_t CHW = static_cast<int64_t>(C) * H * W;
    const int64_t total = static_cast<int64_t>(N) * CHW;
    if (total == 0) return DN_OK;
    if (!input || !output) return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_simple_gate: null pointer");
    const auto* hin = static_cast<const __half*>(input);
    auto* hout = static_cast<__half*>(output);
    if (CHW % 8 == 0 && al16(input) && al16(output))
        gate_kernel<true><<<grid_for(total, kThreads * 8), kThreads, 0, to_stream(stream)>>>(hin, hout, CHW, total);
    else
        gate_kernel<false><<<grid_for(total, kThreads), kThreads, 0, to_stream(stream)>>>(hin, hout, CHW, total);
    return launched("dn_launch_simple_gate");
}

int dn_launch_global_avg_pool(const void* input, void* output, int N, int C, int H, int W, void* stream) {
    const char* name = "dn_launch_global_avg_pool";
    DN_TRY(pool_check(input, output, N, C, H, W, name));
    const PoolPlan pp = pool_plan(input, N, C, H, W);
    if (pp.planes == 0) return DN_OK;
    cudaStream_t s = to_stream(stream);
    void* scratch = nullptr;
    cudaError_t e = cudaMallocAsync(&scratch, static_cast<size_t>(pp.planes) * pp.splits * sizeof(float), s);
    if (e != cudaSuccess) return dn_cuda_fail(e, "dn_launch_global_avg_pool: scratch allocation");
    const int rc = pool_launch(pp, input, output, static_cast<float*>(scratch), s, name);
    e = cudaFreeAsync(scratch, s);
    if (rc != DN_OK) return rc;
    if (e != cudaSuccess) return dn_cuda_fail(e, "dn_launch_global_avg_pool: scratch release");
    return DN_OK;
}

// Same plan and kernels as dn_launch_global_avg_pool; only the scratch
// differs. Nothing in it needs to start at zero: the split kernel writes
// every slot the final kernel reads, in the same call.
int dn_launch_global_avg_pool_noalloc(const void* input, void* output, int N, int C, int H, int W, void* stream) {
    const char* name = "dn_launch_global_avg_pool_noalloc";
    DN_TRY(pool_check(input, output, N, C, H, W, name));
    const PoolPlan pp = pool_plan(input, N, C, H, W);
    if (pp.planes == 0) return DN_OK;
    // The size rule is checked on the host before any CUDA call, so a
    // rejected size touches neither the device nor the runtime.
    const int64_t need = pp.planes * pp.splits;
    if (need > kNoAllocPoolFloats)
        return dn_fail_str(DN_ERR_UNSUPPORTED,
                           std::string(name) + ": N*C*splits = " + std::to_string(need) +
                               " split sums exceed the static scratch of " + std::to_string(kNoAllocPoolFloats) +
                               " floats (splits = min(128, ceil(H*W / 16384)))");
    float* scratch = nullptr;
    DN_TRY(pool_scratch(&scratch, name));
    return pool_launch(pp, input, output, scratch, to_stream(stream), name);
}

int dn_launch_mul_channelwise(const void* input, const void* scale, void* output, int N, int C, int H, int W,
                              void* stream) {
    return run_chan<false>(input, nullptr, scale, false, output, N, C, H, W, stream, "dn_launch_mul_channelwise");
}

int dn_launch_add(const void* a, const void* b, void* out, int64_t n, void* stream) {
    return run_flat<kAdd>(a, b, 0.f, out, n, stream, "dn_launch_add");
}

int dn_launch_mul_scalar(const void* input, float scalar, void* output, int64_t n, void* stream) {
    return run_flat<kMulScalar>(input, nullptr, scalar, output, n, stream, "dn_launch_mul_scalar");
}

int dn_launch_scaled_add(const void* identity, const void* residual, const void* scale, int scale_fp32,
                         void* output, int N, int C, int H, int W, void* stream) {
    return run_chan<true>(identity, residual, scale, scale_fp32 != 0, output, N, C, H, W, stream,
                          "dn_launch_scaled_add");
}

int dn_launch_pixel_shuffle2x(const void* input, void* output, int N, int C_in, int H, int W, void* stream) {
    if (any_negative({N, C_in, H, W})) return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_pixel_shuffle2x: negative size");
    if (C_in % 4 != 0) return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_pixel_shuffle2x: C_in must be divisible by 4");
    const int Cout = C_in / 4;
    const int64_t total = static_cast<int64_t>(N) * Cout * 2 * H * W;  // output pairs
    if (total == 0) return DN_OK;
    if (!input || !output) return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_pixel_shuffle2x: null pointer");
    const auto* hin = static_cast<const __half*>(input);
    auto* hout = static_cast<__half*>(output);
    if (al4(output))
        shuffle_kernel<true><<<grid_for(total, kThreads), kThreads, 0, to_stream(stream)>>>(hin, hout, Cout, H, W,
                                                                                           total);
    else
        shuffle_kernel<false><<<grid_for(total, kThreads), kThreads, 0, to_stream(stream)>>>(hin, hout, Cout, H, W,
                                                                                            total);
    return launched("dn_launch_pixel_shuffle2x");
}

int dn_upsample_bilinear(const void* input, void* output, int N, int C, int H, int W, int scale_factor,
                         void* stream) {
    if (scale_factor <= 0) return dn_fail(DN_ERR_INVALID_ARG, "dn_upsample_bilinear: scale_factor must be > 0");
    if (any_negative({N, C, H, W})) return dn_fail(DN_ERR_INVALID_ARG, "dn_upsample_bilinear: negative size");
    const int64_t Ho = static_cast<int64_t>(H) * scale_factor, Wo = static_cast<int64_t>(W) * scale_factor;
    if (Ho > 0x7fffffff || Wo > 0x7fffffff) return dn_fail(DN_ERR_INVALID_ARG, "dn_upsample_bilinear: output too large");
    const int64_t total = static_cast<int64_t>(N) * C * Ho * Wo;
    if (total == 0) return DN_OK;
    if (!input || !output) return dn_fail(DN_ERR_INVALID_ARG, "dn_upsample_bilinear: null pointer");
    upsample_kernel<<<grid_for(total, kThreads), kThreads, 0, to_stream(stream)>>>(
        static_cast<const __half*>(input), static_cast<__half*>(output), H, W, static_cast<int>(Ho),
        static_cast<int>(Wo), static_cast<float>(scale_factor), total);
    return launched("dn_upsample_bilinear");
}

int dn_launch_warp_bilinear(const void* feat, const void* offset, void* output, int N, int C, int H, int W,
                            void* stream) {
    if (any_negative({N, C, H, W})) return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_warp_bilinear: negative size");
    const int64_t total = static_cast<int64_t>(N) * H * W;
    if (total * C == 0) return DN_OK;
    if (!feat || !offset || !output) return dn_fail(DN_ERR_INVALID_ARG, "dn_launch_warp_bilinear: null pointer");
    warp_kernel<<<grid_for(total, kThreads), kThreads, 0, to_stream(stream)>>>(
        static_cast<const __half*>(feat), static_cast<const __half*>(offset), static_cast<__half*>(output), C, H, W,
        total);
    return launched("dn_launch_warp_bilinear");
}

}  // extern "C"
