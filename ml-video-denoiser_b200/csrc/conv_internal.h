// Internal entry points of the stand-alone convolution layers (conv_layers.cu)
// for engine components that build layers from host arrays and keep their
// feature maps channel-last (NHWC) between layers.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "denoiser_b200_layers.h"

namespace dnb {

// Layers from host FP32 arrays (rounded to FP16 like exported weights);
// bias may be null. Same shape rules and status codes as dn_conv2d_create /
// dn_dcn_create.
int conv2d_build(const float* w, const float* bias, int cout, int cin_g, int kh, int kw, int pad, int stride,
                 int dilation, int groups, int device, dn_conv2d** out);
int dcn_build(const float* w, const float* bias, int cout, int cin, int kh, int kw, int pad, int stride, int dilation,
              int deform_groups, int device, dn_dcn** out);

// Forward from an NHWC input (no transpose); output NCHW, or NHWC with out_nhwc.
int conv2d_run_nhwc(dn_conv2d* L, const __half* x_nhwc, int N, int H, int W, void* out, bool out_nhwc,
                    cudaStream_t s);
int conv2d_to_nhwc(const __half* in, __half* out, int N, int C, int HW, cudaStream_t s);

// The fusion epilogue of a batch-1 deformable conv: instead of storing its
// Cout channels, acc[j][pix] += sum_o w[j][o] * out[o][pix] for j < 3 (FP32
// planes); with out16 set, the sum is written there as FP16 planes instead.
// w is [3][dcn_nt(L)] (zero padded past Cout).
struct DcnFuse {
    const float* w;
    float* acc;
    __half* out16;
};
int dcn_nt(const dn_dcn* L);

// Deformable conv from an NHWC input; offsets = off (+ off2), raw masks = msk
// (+ msk2), each term FP16 in the layer's layout, summed in FP32.
int dcn_run_nhwc(dn_dcn* L, const __half* x_nhwc, const __half* off, const __half* msk, const __half* off2,
                 const __half* msk2, int N, int H, int W, void* out, const DcnFuse* fuse, cudaStream_t s);

// Read and clear a layer's device error word.
int conv2d_check(dn_conv2d* L);
int dcn_check(dn_dcn* L);

}  // namespace dnb
