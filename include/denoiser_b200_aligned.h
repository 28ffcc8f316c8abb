/*
 * denoiser_b200_aligned.h — C-ABI of the temporal NAFNet with deformable
 * alignment (FP16, batch 1, 3-channel frames).
 *
 * No model of the reference uses its DeformConv2dLayer
 * (src/layers/deform_conv2d.cu:105-184); this model fixes one wiring around
 * it and runs it inside a whole network:
 *   f_t   = feat(frame_t)                        3x3 conv, 3 -> F
 *   om_t  = offset(concat(f_c, f_t))             3x3 conv, 2F -> 3*dg*9
 *           (2*dg*9 offsets [dy, dx] per (group, tap), then dg*9 raw masks)
 *   a_t   = DeformConv2d(f_t, offsets, masks)    3x3, F -> F, sigmoid masks
 *   a_c   = f_c                                  c = T / 2
 *   fused = fuse(concat(a_0 .. a_{T-1})) + frame_c   1x1 conv, T*F -> 3
 *   y     = NAFNet(fused)                        the spatial engine (trunk)
 * Weights: manifest keys align.{feat,offset,dcn,fuse}.{weight,bias} in the
 * reference format (architecture num_frames = T), and a separate spatial
 * NAFNet manifest for the trunk.
 *
 * Frame cache (like dn_model_encode_frame / dn_model_decode_window): a
 * sequence encodes each frame once into slot f % T, and each output decodes
 * the window whose frame t sits in slots[t] (edge replication = a repeated
 * slot). The slots hold the frame, its features and its share of the offset
 * conv; they stay valid while the frame size does not change (a new size
 * synchronises the stream and reallocates them).
 *
 * Calls for one model come from one host thread; all work is asynchronous on
 * `stream` (a cudaStream_t; NULL = legacy default stream).
 */
#ifndef DENOISER_B200_ALIGNED_H
#define DENOISER_B200_ALIGNED_H

#include "denoiser_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct dn_aligned dn_aligned;

/* Load the alignment weights and the trunk NAFNet onto `device`.
 * DN_ERR_IO / DN_ERR_FORMAT / DN_ERR_NOT_FOUND as dn_model_create;
 * DN_ERR_UNSUPPORTED for frames other than 3 channels or F not in
 * {32, 64, 128}. */
int dn_aligned_create(const char* align_manifest, const char* trunk_manifest, int device, dn_aligned** out);
int dn_aligned_destroy(dn_aligned* model);
int dn_aligned_info(const dn_aligned* model, int* num_frames, int* in_channels, int* feat_channels,
                    int* deform_groups);

/* Encode one (1, 3, H, W) FP16 NCHW device frame into `slot` in [0, T). */
int dn_aligned_encode_frame(dn_aligned* model, const void* frame, int H, int W, int slot, void* stream);

/* The alignment stage alone: the trunk input `fused` (1, 3, H, W) FP16 of the
 * window slots[0 .. T-1] (T must equal num_frames). */
int dn_aligned_align_window(dn_aligned* model, const int* slots, int T, void* fused, void* stream);

/* Alignment and trunk: y (1, 3, H, W) FP16 for the window slots[0 .. T-1]. */
int dn_aligned_decode_window(dn_aligned* model, const int* slots, int T, void* y, void* stream);

/* One window without the cache: clip (1, T, 3, H, W) FP16 NCHW -> y. */
int dn_aligned_forward(dn_aligned* model, const void* clip, int H, int W, void* y, void* stream);

/* Synchronise `stream`; DN_ERR_DEVICE if a kernel reported a device error. */
int dn_aligned_sync(dn_aligned* model, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* DENOISER_B200_ALIGNED_H */
