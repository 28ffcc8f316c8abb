// Pixel-unit bilinear warp of NHWC features for the temporal model of the
// reference C++ engine (warp_bilinear_kernel, src/kernels/nafnet_kernels.cu
// :212-262): out(y, x) = bilinear(feat, x + dx, y + dy), every tap clamped
// to the border, offsets ch0 = dx, ch1 = dy. One thread = one pixel x 8
// channels (16-byte vectors).
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
                                  int C) {
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
    const float fx = static_cast<float>(x) + __half2float(o[0]);
    const float fy = static_cast<float>(y) + __half2float(o[1]);
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

}  // namespace

int launch_warp_pixel(const __half* feat, const __half* off, int off_stride, __half* out, int nimg,
                      int H, int W, int C, cudaStream_t s) {
    if (C % 8 != 0) return dn_fail(DN_ERR_UNSUPPORTED, "warp: channels must be a multiple of 8");
    const long long total = static_cast<long long>(nimg) * H * W * (C / 8);
    const int blocks = static_cast<int>((total + 255) / 256);
    cudaError_t e = launch_pdl(warp_pixel_kernel, dim3(blocks), dim3(256), 0, s, feat, off, off_stride, out, nimg, H, W, C);
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "warp: launch");
}

}  // namespace dnb
