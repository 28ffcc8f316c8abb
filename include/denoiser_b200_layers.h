/*
 * denoiser_b200_layers.h — C-ABI of the stand-alone convolution layers of the
 * reference's include/denoiser/layers/ (the model forwards use the engine).
 *
 * Tensors are device pointers to FP16 NCHW data; `stream` is a cudaStream_t
 * (NULL = legacy default stream). Every function returns DN_OK or a negative
 * DN_ERR_* code (denoiser_b200.h); dn_last_error() has the message.
 */
#ifndef DENOISER_B200_LAYERS_H
#define DENOISER_B200_LAYERS_H

#include "denoiser_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------
 * DeformConv2dLayer (include/denoiser/layers/deform_conv2d.h:11-55):
 * modulated deformable convolution (DCNv2). offsets (N, 2*dg*kH*kW, Ho, Wo)
 * hold (dy, dx) per (deform group, tap); masks (N, dg*kH*kW, Ho, Wo) are raw
 * (the sigmoid is applied inside). One fused kernel samples and multiplies on
 * the tensor cores (FP32 accumulation; the reference accumulates in FP16).
 * ------------------------------------------------------------------------ */
typedef struct dn_dcn dn_dcn;

/* DeformConv2dLayer(store, weight_name, bias_name, pad, stride, dilation,
 * deform_groups) (deform_conv2d.cu:76-98): weight (Cout, Cin, kH, kW), bias
 * (Cout) from the store, packed and uploaded to `device`. bias_name may be
 * NULL (no bias). DN_ERR_NOT_FOUND for a missing key (std::out_of_range in
 * the reference), DN_ERR_FORMAT for a non-4-D weight, DN_ERR_UNSUPPORTED for
 * Cout > 256 or Cin/deform_groups not dividing 64. */
int dn_dcn_create(const dn_weights* store, const char* weight_name, const char* bias_name, int pad, int stride,
                  int dilation, int deform_groups, int device, dn_dcn** out);
int dn_dcn_destroy(dn_dcn* layer);
/* out_channels() / in_channels() / deform_groups() and the kernel size. */
int dn_dcn_info(const dn_dcn* layer, int* out_channels, int* in_channels, int* deform_groups, int* kernel_h,
                int* kernel_w);
/* Output spatial size for an input of H_in x W_in. */
int dn_dcn_output_size(const dn_dcn* layer, int H_in, int W_in, int* H_out, int* W_out);
/* DeformConv2dLayer::forward (deform_conv2d.cu:105-184) into `output`
 * (N, Cout, Ho, Wo), asynchronous on `stream`. The layer keeps an NHWC copy
 * of the input (grown on demand), so calls on one layer must not overlap. */
int dn_dcn_forward(dn_dcn* layer, const void* input, const void* offsets, const void* masks, int N, int H_in,
                   int W_in, void* output, void* stream);
/* Synchronise `stream` and report a device-side error of the layer's kernel. */
int dn_dcn_sync(dn_dcn* layer, void* stream);

/* ------------------------------------------------------------------------
 * Conv2dLayer (include/denoiser/layers/conv2d.h:44-63): regular convolution
 * with symmetric zero padding, stride, dilation and groups, weight
 * (Cout, Cin/groups, kH, kW) and optional bias (Cout) from the store. One
 * implicit-GEMM kernel on the tensor cores per 256 output channels (FP32
 * accumulation), bias fused; the reference runs cuDNN plus a bias pass.
 * ------------------------------------------------------------------------ */
typedef struct dn_conv2d dn_conv2d;

/* Conv2dLayer(store, weight_name, bias_name, pad, stride, dilation, groups)
 * (src/layers/conv2d.cu:16-92); bias_name NULL = std::nullopt. Errors as for
 * dn_dcn_create (DN_ERR_INVALID_ARG when Cout is not divisible by groups). */
int dn_conv2d_create(const dn_weights* store, const char* weight_name, const char* bias_name, int pad, int stride,
                     int dilation, int groups, int device, dn_conv2d** out);
int dn_conv2d_destroy(dn_conv2d* layer);
/* out_channels(), in_channels() (= weight dim 1, per group), kernel_h(),
 * kernel_w(), groups(). */
int dn_conv2d_info(const dn_conv2d* layer, int* out_channels, int* in_channels, int* kernel_h, int* kernel_w,
                   int* groups);
int dn_conv2d_output_size(const dn_conv2d* layer, int H_in, int W_in, int* H_out, int* W_out);
/* Conv2dLayer::forward (conv2d.cu:94-150): input (N, C, H, W) with
 * C = in_channels * groups -> output (N, Cout, Ho, Wo), asynchronous on
 * `stream`; calls on one layer must not overlap (the layer keeps an NHWC
 * copy of the input). */
int dn_conv2d_forward(dn_conv2d* layer, const void* input, int N, int C, int H_in, int W_in, void* output,
                      void* stream);
int dn_conv2d_sync(dn_conv2d* layer, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DENOISER_B200_LAYERS_H */
