/*
 * denoiser_b200_infer.h — frame-level inference helpers (device buffers,
 * asynchronous on `stream`), the kernels behind tiled inference with ramp
 * blending and temporal flip averaging of the reference's training/infer.py:
 *
 *   tile grid:  overlap = tile / 8, stride = tile - overlap, tiles start at
 *               0, stride, 2*stride, ... and are clipped to the frame
 *               (_tile_inference, infer.py:174-203; the temporal form
 *               _tile_inference_temporal, :318-346, tiles every frame of the
 *               clip alike);
 *   blending:   acc += pred * ramp_y[y] * ramp_x[x], wsum += ramp_y * ramp_x,
 *               out = acc / max(wsum, 1e-6) (_make_ramp, :206-216);
 *   flip:       final = (forward + backward) * 0.5
 *               (denoise_temporal_sequence, :219-274).
 */
#ifndef DENOISER_B200_INFER_H
#define DENOISER_B200_INFER_H

#include "denoiser_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* dst (planes, th, tw) FP16 = src (planes, H, W)[:, y0:y0+th, x0:x0+tw]. */
int dn_tile_extract(const void* src, void* dst, int64_t planes, int H, int W, int y0, int x0, int th, int tw,
                    void* stream);
/* acc (C, H, W) FP32 and wsum (H, W) FP32 += the ramp-weighted tile
 * pred (C, th, tw) FP16 placed at (y0, x0). DN_ERR_INVALID_ARG when the tile
 * is narrower than `overlap` along an axis (the reference's ramp assignment
 * fails there too). */
int dn_tile_accumulate(const void* pred, float* acc, float* wsum, int C, int H, int W, int y0, int x0, int th, int tw,
                       int overlap, void* stream);
/* out (C, H, W) FP16 = acc / max(wsum, 1e-6). */
int dn_tile_normalize(const float* acc, const float* wsum, void* out, int C, int H, int W, void* stream);
/* out[i] = (a[i] + b[i]) * 0.5 in FP32, stored FP16 (n elements). */
int dn_average_pair(const void* a, const void* b, void* out, int64_t n, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* DENOISER_B200_INFER_H */
