/*
 * denoiser_b200.h — C-ABI of the B200 NAFNet denoiser engine.
 *
 * This is the drop-in boundary: plain C types only (pointers, ints, sizes,
 * an opaque stream handle that is a cudaStream_t). Every function returns
 * DN_OK (0) or a negative DN_ERR_* code; dn_last_error() gives the calling
 * thread's message for the last failure. Nothing here throws.
 *
 * The C++ API in include/denoiser/ (Tensor, WeightStore, Conv2dLayer, NAFNet,
 * NAFNetTemporal, kernels::launch_*) is a source-compatible mirror of the
 * reference engine's include/denoiser/ headers, implemented on top of these
 * entry points; it maps the codes back to the reference's exception types:
 *   DN_ERR_IO / DN_ERR_FORMAT / DN_ERR_DTYPE / DN_ERR_CUDA -> std::runtime_error
 *   DN_ERR_NOT_FOUND                                        -> std::out_of_range
 *   DN_ERR_INVALID_ARG                                      -> std::invalid_argument
 */
#ifndef DENOISER_B200_H
#define DENOISER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DN_OK 0
#define DN_ERR_INVALID_ARG -1 /* bad pointer / shape / parameter            */
#define DN_ERR_CUDA -2        /* a CUDA runtime call failed                  */
#define DN_ERR_IO -3          /* manifest or .bin missing / unreadable       */
#define DN_ERR_FORMAT -4      /* malformed manifest, .bin size != shape      */
#define DN_ERR_NOT_FOUND -5   /* weight key not in the manifest              */
#define DN_ERR_UNSUPPORTED -6 /* shape or architecture this build rejects    */
#define DN_ERR_DEVICE -7      /* a kernel reported a device-side error       */
#define DN_ERR_DTYPE -8       /* tensor of the wrong dtype (e.g. FP32 input) */

/* Message of the calling thread's most recent failure ("" if none). */
const char* dn_last_error(void);

/* ABI version of this library (major * 100 + minor). */
int dn_abi_version(void);

/*
 * Descriptor self-check of the tcgen05 path (no reference counterpart):
 * D[128 x N] = A[128 x K] * B[N x K]^T on one CTA, fp16 in, fp32 out.
 * All pointers are device pointers; err_dev receives a device error word.
 */
int dn_umma_probe(const void* A, const void* B, float* D, int N, int K, uint32_t* err_dev,
                  void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* DENOISER_B200_H */
