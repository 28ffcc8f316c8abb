// Temporal-model kernels on NHWC features.
//
// warp_pixel_kernel: bilinear warp, out(y, x) = bilinear(feat, x + sx*dx,
//   y + sy*dy), every tap clamped to the border, offsets ch0 = dx, ch1 = dy.
//   sx = sy = 1 is the C++ engine's warp_bilinear_kernel
//   (src/kernels/nafnet_kernels.cu:212-262); sx = (W-1)/W, sy = (H-1)/H is
//   the PyTorch model's _warp (training/models.py:321-343: grid_sample with
//   align_corners=True and border padding, offsets normalised by W/2, H/2),
//   since clamping the sample point and clamping each tap give the same value.
//   One thread = one pixel x 8 channels (16-byte vectors).
// dw_pair_kernel: depthwise 3x3 (zero padding, no bias) over the channel
//   concatenation [a, b] of two C-channel maps: the first layer of an offset
//   head (_make_offset_head, training/models.py:346-372).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kernels.h"
#include "launch.cuh"
#include "sm100.cuh"
#include "status.h"

namespace dnb {
namespace {

__global__ void warp_pixel_kernel(const __half* __restrict__ feat, const __half* __restrict__ off,
                                  int off_stride, __half* __restrict__ out, int nimg, int H, int W,
                                  int C, float sx, float sy) {
    pdl_trigger();
    pdl_wait();
    const int groups = C / 8;
    const long long total = static_cast<long long>(nimg) * H * W * groups;
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int g = static_cast<int>(i % groups);
    const long long pixg = i / groups;
    const int x = static_cast<int>(pixg % W);
    const int y = static_cast<int>((pixg / W) % H);
    const long long img = pixg / (static_cast<long long>(H) * W);
    const __half* o = off + pixg * off_stride;
    const float fx = static_cast<float>(x) + sx * __half2float(o[0]);
    const float fy = static_cast<float>(y) + sy * __half2float(o[1]);
    const float x0f = floorf(fx), y0f = floorf(fy);
    const float wx = fx - x0f, wy = fy - y0f;
    const int x0 = static_cast<int>(x0f), y0 = static_cast<int>(y0f);
    const __half* base = feat + img * H * W * C + g * 8;
    auto tap = [&](int yy, int xx, float w, float (&acc)[8]) {
        yy = min(max(yy, 0), H - 1);
        xx = min(max(xx, 0), W - 1);
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(base + (static_cast<size_t>(yy) * W + xx) * C));
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 t = unpack_half2(u[k]);
            acc[2 * k] += w * t.x;
            acc[2 * k + 1] += w * t.y;
        }
    };
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    tap(y0, x0, (1.f - wy) * (1.f - wx), acc);
    tap(y0, x0 + 1, (1.f - wy) * wx, acc);
    tap(y0 + 1, x0, wy * (1.f - wx), acc);
    tap(y0 + 1, x0 + 1, wy * wx, acc);
    uint4 r;
    r.x = pack_half2(acc[0], acc[1]);
    r.y = pack_half2(acc[2], acc[3]);
    r.z = pack_half2(acc[4], acc[5]);
    r.w = pack_half2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + pixg * C + g * 8) = r;
}

__global__ void __launch_bounds__(256) dw_pair_kernel(const __half* __restrict__ a, const __half* __restrict__ b,
                                                      const float* __restrict__ w, __half* __restrict__ out, int H,
                                                      int W, int C) {
    pdl_trigger();
    const int groups = 2 * C / 8;
    const long long total = static_cast<long long>(H) * W * groups;
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int g = static_cast<int>(i % groups);
    const int c = g * 8;  // channel of the concatenation
    float tw[9][8];
#pragma unroll
    for (int t = 0; t < 9; ++t)
#pragma unroll
        for (int k = 0; k < 8; ++k) tw[t][k] = w[t * 2 * C + c + k];
    pdl_wait();
    if (i >= total) return;
    const long long pix = i / groups;
    const int x = static_cast<int>(pix % W);
    const int y = static_cast<int>(pix / W);
    const __half* src = c < C ? a + c : b + (c - C);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int ky = 0; ky < 3; ++ky) {
        const int yy = y + ky - 1;
        if (yy < 0 || yy >= H) continue;
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
            const int xx = x + kx - 1;
            if (xx < 0 || xx >= W) continue;
            float f[8];
            h8_to_f(*reinterpret_cast<const uint4*>(src + (static_cast<long long>(yy) * W + xx) * C), f);
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[k] = fmaf(f[k], tw[ky * 3 + kx][k], acc[k]);
        }
    }
    *reinterpret_cast<uint4*>(out + pix * 2 * C + c) = f_to_h8(acc);
}

}  // namespace

int launch_dw_pair(const __half* a, const __half* b, const float* w, __half* out, int H, int W, int C, cudaStream_t s) {
    if (C % 8 != 0) return dn_fail(DN_ERR_UNSUPPORTED, "offset head: channels must be a multiple of 8");
    const long long total = static_cast<long long>(H) * W * (2 * C / 8);
    const int blocks = static_cast<int>((total + 255) / 256);
    cudaError_t e = launch_pdl(dw_pair_kernel, dim3(blocks), dim3(256), 0, s, a, b, w, out, H, W, C);
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "offset head depthwise: launch");
}

int launch_warp_pixel(const __half* feat, const __half* off, int off_stride, __half* out, int nimg,
                      int H, int W, int C, float sx, float sy, cudaStream_t s) {
    if (C % 8 != 0) return dn_fail(DN_ERR_UNSUPPORTED, "warp: channels must be a multiple of 8");
    const long long total = static_cast<long long>(nimg) * H * W * (C / 8);
    const int blocks = static_cast<int>((total + 255) / 256);
    cudaError_t e = launch_pdl(warp_pixel_kernel, dim3(blocks), dim3(256), 0, s, feat, off, off_stride, out, nimg, H, W,
                               C, sx, sy);
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "warp: launch");
}

}  // namespace dnb
