// Frame-level inference helpers of the engine: tiled inference with linear
// ramp blending and the average of two passes (temporal flip averaging), as
// in the reference's training/infer.py:
//   _tile_inference / _tile_inference_temporal (:174-203, 318-346): tiles of
//     tile_size with overlap = tile_size / 8 and stride = tile_size - overlap;
//     output += pred * ramp and weights += ramp over each tile, then
//     output / max(weights, 1e-6);
//   _make_ramp (:206-216): per axis ones, the first `overlap` entries set to
//     linspace(0, 1, overlap), then the last `overlap` entries to its
//     reverse (the second assignment wins where they overlap); the tile's
//     weight is ramp_y[y] * ramp_x[x];
//   denoise_temporal_sequence (:219-274): final = (forward + backward) * 0.5.
// The blending runs on FP32 planes in device memory; the tile extraction
// copies a window of a planar tensor so the model sees a contiguous tile.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <string>

#include "denoiser_b200_infer.h"
#include "status.h"

namespace dnb {
namespace {

constexpr int kT = 256;

// Entry i of the ramp of an axis of length n (see the file comment).
__device__ __forceinline__ float ramp_at(int i, int n, int overlap) {
    if (overlap <= 0) return 1.f;
    auto lin = [overlap](int k) { return overlap == 1 ? 0.f : static_cast<float>(k) / static_cast<float>(overlap - 1); };
    float r = 1.f;
    if (i < overlap) r = lin(i);
    if (i >= n - overlap) r = lin(n - 1 - i);
    return r;
}

__global__ void __launch_bounds__(kT) extract_kernel(const __half* __restrict__ src, __half* __restrict__ dst,
                                                     int64_t planes, int H, int W, int y0, int x0, int th, int tw) {
    const int64_t total = planes * th * tw;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kT + threadIdx.x; i < total; i += static_cast<int64_t>(gridDim.x) * kT) {
        const int x = static_cast<int>(i % tw);
        const int64_t r = i / tw;
        const int y = static_cast<int>(r % th);
        const int64_t p = r / th;
        dst[i] = src[(p * H + y0 + y) * W + x0 + x];
    }
}

__global__ void __launch_bounds__(kT) accumulate_kernel(const __half* __restrict__ pred, float* __restrict__ acc,
                                                        float* __restrict__ wsum, int C, int H, int W, int y0, int x0,
                                                        int th, int tw, int overlap) {
    const int64_t px = static_cast<int64_t>(th) * tw;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kT + threadIdx.x; i < px; i += static_cast<int64_t>(gridDim.x) * kT) {
        const int x = static_cast<int>(i % tw), y = static_cast<int>(i / tw);
        const float w = ramp_at(y, th, overlap) * ramp_at(x, tw, overlap);
        const int64_t o = static_cast<int64_t>(y0 + y) * W + x0 + x;
        for (int c = 0; c < C; ++c) acc[c * static_cast<int64_t>(H) * W + o] += __half2float(pred[c * px + i]) * w;
        wsum[o] += w;
    }
}

__global__ void __launch_bounds__(kT) normalize_kernel(const float* __restrict__ acc, const float* __restrict__ wsum,
                                                       __half* __restrict__ out, int C, int64_t HW) {
    const int64_t total = C * HW;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kT + threadIdx.x; i < total; i += static_cast<int64_t>(gridDim.x) * kT)
        out[i] = __float2half(acc[i] / fmaxf(wsum[i % HW], 1e-6f));
}

__global__ void __launch_bounds__(kT) average_kernel(const __half* __restrict__ a, const __half* __restrict__ b,
                                                     __half* __restrict__ out, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kT + threadIdx.x; i < n; i += static_cast<int64_t>(gridDim.x) * kT)
        out[i] = __float2half((__half2float(a[i]) + __half2float(b[i])) * 0.5f);
}

unsigned grid_of(int64_t n) {
    const int64_t g = (n + kT - 1) / kT;
    return static_cast<unsigned>(g < 148 * 16 ? (g > 0 ? g : 1) : 148 * 16);
}

int launched(const char* name) {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, name);
}

}  // namespace
}  // namespace dnb

using namespace dnb;

extern "C" {

int dn_tile_extract(const void* src, void* dst, int64_t planes, int H, int W, int y0, int x0, int th, int tw,
                    void* stream) {
    if (!src || !dst) return dn_fail(DN_ERR_INVALID_ARG, "dn_tile_extract: null pointer");
    if (planes <= 0 || th <= 0 || tw <= 0 || y0 < 0 || x0 < 0 || y0 + th > H || x0 + tw > W)
        return dn_fail(DN_ERR_INVALID_ARG, "dn_tile_extract: tile outside the frame");
    extract_kernel<<<grid_of(planes * th * tw), kT, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(src), static_cast<__half*>(dst), planes, H, W, y0, x0, th, tw);
    return launched("dn_tile_extract");
}

int dn_tile_accumulate(const void* pred, float* acc, float* wsum, int C, int H, int W, int y0, int x0, int th, int tw,
                       int overlap, void* stream) {
    if (!pred || !acc || !wsum) return dn_fail(DN_ERR_INVALID_ARG, "dn_tile_accumulate: null pointer");
    if (C <= 0 || th <= 0 || tw <= 0 || y0 < 0 || x0 < 0 || y0 + th > H || x0 + tw > W || overlap < 0)
        return dn_fail(DN_ERR_INVALID_ARG, "dn_tile_accumulate: tile outside the frame");
    // The reference's _make_ramp assigns `overlap` values into an axis of the
    // tile's length and fails when the tile is shorter than that.
    if (overlap > th || overlap > tw)
        return dn_fail_str(DN_ERR_INVALID_ARG, "dn_tile_accumulate: a " + std::to_string(th) + "x" + std::to_string(tw) +
                                                   " tile is narrower than the blend overlap " + std::to_string(overlap));
    accumulate_kernel<<<grid_of(static_cast<int64_t>(th) * tw), kT, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(pred), acc, wsum, C, H, W, y0, x0, th, tw, overlap);
    return launched("dn_tile_accumulate");
}

int dn_tile_normalize(const float* acc, const float* wsum, void* out, int C, int H, int W, void* stream) {
    if (!acc || !wsum || !out) return dn_fail(DN_ERR_INVALID_ARG, "dn_tile_normalize: null pointer");
    if (C <= 0 || H <= 0 || W <= 0) return dn_fail(DN_ERR_INVALID_ARG, "dn_tile_normalize: empty frame");
    const int64_t HW = static_cast<int64_t>(H) * W;
    normalize_kernel<<<grid_of(C * HW), kT, 0, static_cast<cudaStream_t>(stream)>>>(acc, wsum,
                                                                                      static_cast<__half*>(out), C, HW);
    return launched("dn_tile_normalize");
}

int dn_average_pair(const void* a, const void* b, void* out, int64_t n, void* stream) {
    if (n == 0) return DN_OK;
    if (!a || !b || !out || n < 0) return dn_fail(DN_ERR_INVALID_ARG, "dn_average_pair: bad argument");
    average_kernel<<<grid_of(n), kT, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(a), static_cast<const __half*>(b), static_cast<__half*>(out), n);
    return launched("dn_average_pair");
}

}  // extern "C"
