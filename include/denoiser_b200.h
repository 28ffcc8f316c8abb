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

/* ------------------------------------------------------------------------
 * Weights (host half of WeightStore, include/denoiser/weight_loader.h:61-101
 * of the reference; format of training/export.py:48-118). Every .bin is
 * memory-mapped and its size checked against numel * sizeof(dtype).
 * ------------------------------------------------------------------------ */

typedef struct dn_weights dn_weights;

/* WeightStore::WeightStore (weight_loader.cc:63-76): DN_ERR_IO if the
 * manifest or a .bin is missing, DN_ERR_FORMAT for bad JSON, an unknown
 * dtype or a .bin whose size does not match its shape. */
int dn_weights_open(const char* manifest_path, dn_weights** out);
void dn_weights_close(dn_weights* weights);
/* Number of manifest layers (Manifest::layers.size()). */
int dn_weights_count(const dn_weights* weights);
/* WeightStore::contains (weight_loader.h:76): 1 or 0. */
int dn_weights_contains(const dn_weights* weights, const char* name);
/* Shape (up to 8 dims), dtype (0 float32, 1 float16) and the mapped host
 * bytes of `name`; DN_ERR_NOT_FOUND like WeightStore::get's out_of_range. */
int dn_weights_info(const dn_weights* weights, const char* name, int64_t* shape, int* ndim, int* dtype,
                    const void** host_data);
/* Name of layer `index` in manifest order. */
int dn_weights_name(const dn_weights* weights, int index, const char** name);
/* Manifest::Architecture fields (weight_loader.h:30-39). */
int dn_weights_arch(const dn_weights* weights, char* type_buf, int type_buf_len, int* base_channels,
                    int* num_levels, int* in_channels, int* num_frames, int* use_warp);
/* Manifest::version and default dtype (0 float32, 1 float16), the
 * architecture's enc_channels (up to max_enc, count in *n_enc) and
 * out_channels. Strings stay valid until dn_weights_close. */
int dn_weights_meta(const dn_weights* weights, const char** version, int* dtype, int* enc_channels, int max_enc,
                    int* n_enc, int* out_channels);
/* LayerEntry::file of `name` (relative to the manifest directory). */
int dn_weights_file(const dn_weights* weights, const char* name, const char** file);
/* Path of the manifest the store was opened from. */
const char* dn_weights_path(const dn_weights* weights);

/* ------------------------------------------------------------------------
 * Models: NAFNet (spatial) and NAFNetTemporal, architecture discovered from
 * the manifest keys like the reference engine (src/models/nafnet.cu:78-92,
 * 281-333; src/models/nafnet_temporal.cu:260-356). One model = one device;
 * drive each model from one host thread (the reference's contract).
 * ------------------------------------------------------------------------ */

typedef struct dn_model dn_model;

typedef struct dn_model_info {
    int kind;            /* 0 NAFNet, 1 NAFNetTemporal (C++ engine design), 2 NAFNetTemporal (PyTorch design: bottleneck_mix, temporal_mix.N.0, 3-layer offset heads) */
    int in_channels;     /* NAFNet::in_channels()                           */
    int num_levels;      /* NAFNet::num_levels()                            */
    int base_channels;
    int num_frames;      /* NAFNetTemporal::num_frames() (1 for NAFNet)      */
    int use_warp;        /* NAFNetTemporal::use_warp()                      */
    int enc_channels[8]; /* NAFNet::enc_channels(), zero-filled              */
} dn_model_info;

/* Load manifest.json + .bin weights (replaces WeightStore + NAFNet /
 * NAFNetTemporal construction, include/denoiser/models/nafnet.h:13,
 * nafnet_temporal.h:13) and upload them, packed, to `device`.
 * Errors: DN_ERR_IO (missing file), DN_ERR_FORMAT (bad JSON, size or shape),
 * DN_ERR_NOT_FOUND (missing key), DN_ERR_INVALID_ARG (bad device). */
int dn_model_create(const char* manifest_path, int device, dn_model** out);
int dn_model_destroy(dn_model* model);
int dn_model_get_info(const dn_model* model, dn_model_info* info);

/* Forward on device buffers, asynchronous on `stream` (cudaStream_t, NULL =
 * legacy default stream). Replaces NAFNet::forward (nafnet.h:20) for
 * x = (N, C, H, W) fp16 NCHW and NAFNetTemporal::forward (nafnet_temporal.h:20)
 * for x = (N, T, C, H, W); y = (N, 3, H, W) fp16 NCHW (caller-allocated).
 * y = beauty + residual, no clamping (training/models.py:575-577). */
int dn_model_forward(dn_model* model, const void* x, const int64_t* shape, int ndim, void* y,
                     void* stream);

/* Same with host buffers (pinned for full speed): H2D copy, forward, D2H
 * copy, then synchronises `stream` and checks the device error word. This is
 * the CLI's per-frame call (cli/main.cc:300-315 of the reference). */
int dn_model_forward_host(dn_model* model, const void* x_host, const int64_t* shape, int ndim,
                          void* y_host, void* stream);

/* Pipelined form of dn_model_forward_host for frame streams (no reference
 * counterpart): enqueues the input copy, the forward and the output copy
 * and returns without waiting. The forward runs on `stream` after the work
 * already queued there; the copies run on two streams of the model, so the
 * input copy of the next call and the output copy of the previous call
 * overlap this call's forward (two staging buffer pairs on the device). The
 * host buffers must stay untouched until the call has completed, and y_host
 * holds the result only after dn_model_host_join(model, s) followed by a
 * synchronisation of `s` (dn_model_sync). Pinned host buffers are needed for
 * the copies to overlap anything. Calls for one model must come from one
 * host thread and use one stream. */
int dn_model_forward_host_async(dn_model* model, const void* x_host, const int64_t* shape, int ndim,
                                void* y_host, void* stream);
/* Makes `stream` wait for the output copies of every dn_model_forward_host_async
 * call issued so far (asynchronous; no host wait). */
int dn_model_host_join(dn_model* model, void* stream);

/* Temporal models over a frame sequence with a frame cache (no reference
 * counterpart: the reference CLI rebuilds and re-encodes a T-frame clip for
 * every output frame, cli/main.cc:260-267). The model keeps the encoder
 * features of T frames in slots 0 .. T-1:
 *   dn_model_encode_frame  runs the encoder on one (1, C, H, W) frame into
 *                          `slot`;
 *   dn_model_decode_window denoises the window whose frame t sits in
 *                          slots[t] (edge replication = a repeated slot),
 *                          with `beauty` = the (1, C, H, W) reference frame,
 *                          into y (1, 3, H, W).
 * A sequence then encodes every frame once (frame f in slot f % T) instead of
 * T times. The slots stay valid while the frame size does not change.
 * DN_ERR_INVALID_ARG for spatial models or slots outside [0, T). */
int dn_model_encode_frame(dn_model* model, const void* frame, int C, int H, int W, int slot, void* stream);
int dn_model_decode_window(dn_model* model, const int* slots, int T, const void* beauty, int C, int H, int W,
                           void* y, void* stream);

/* Synchronise `stream`; DN_ERR_DEVICE if a kernel reported a device-side
 * error (e.g. a bounded wait that expired) since the last check. */
int dn_model_sync(dn_model* model, void* stream);

/* Device bytes of the packed weights and the activation arena of the last
 * planned shape, and the number of kernels the last forward launched. */
int dn_model_stats(const dn_model* model, size_t* weight_bytes, size_t* activation_bytes,
                   int* kernels_per_forward);

/* Select the fused NAFBlock kernels (default 1): both passes for blocks with
 * <= 64 channels (the first pass of 32/64-channel blocks as one tensor-core
 * 3x3 conv of the normalised input), the single-kernel second pass for 128-
 * and 256-channel blocks of a single-image forward, the ending conv of a
 * 32/64-channel model on the tensor cores; 3: the same with the first pass
 * of single images as conv1 on the tensor cores and the depthwise conv on the
 * CUDA cores (a slower alternative kept for comparison); 4: the same as 1
 * with the 1x1-conv GEMMs of 128/256-wide tiles on CTA pairs (cta_group::2
 * MMAs, each CTA loading half of every B tile; also slower, kept for
 * comparison); 2: the first pass (LN, conv1 MMA, depthwise taps) and the
 * ending on the CUDA cores; 0: the per-conv kernels everywhere. Results agree
 * within the parity tolerance; the switch exists for testing every path. */
int dn_model_set_fused(dn_model* model, int enable);

/* Per-launch CUDA-event timing of the engine's kernels (no reference
 * counterpart; the reference engine has no timers). While enabled, every
 * kernel the model launches is bracketed by events on its stream.
 * enable: 0 off, 1 report per kernel kind, 2 per kind and shape
 * ("kind@shape", e.g. the GEMM's M/N/K or the block's width and size). */
int dn_model_profile(dn_model* model, int enable);
/* Synchronise and write a JSON object {kind: {launches, ms, bytes, flops}}
 * accumulated since the previous report (bytes/flops are algorithmic). */
int dn_model_profile_report(dn_model* model, char* buf, size_t len);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* DENOISER_B200_H */
