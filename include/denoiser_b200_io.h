/*
 * denoiser_b200_io.h — image file codecs of the denoiser CLI (host only).
 *
 * The reference reads and writes PNG/JPEG through stb and EXR through
 * tinyexr (src/io/image_io.cc:69-135, src/io/exr_io.cc:29-213), neither of
 * which ships with it (empty submodules). These entry points replace them
 * with this library's own codecs, with the reference's pixel semantics:
 *   PNG  8/16-bit gray, gray+alpha, RGB, RGBA, 8-bit palette; loads as 3
 *        channels, value / 255 (16-bit: high byte); saves 8-bit,
 *        clamp(v * 255 + 0.5);
 *   EXR  single-part scanline, HALF/FLOAT/UINT, NONE/RLE/ZIPS/ZIP; loads
 *        R,G,B (else Y, else the first channel); saves 1 (Y) or 3 (B,G,R)
 *        HALF channels, ZIP;
 *   PPM  binary P5/P6 (8/16-bit) and PFM (PF/Pf, little-endian) as extras.
 * JPEG returns DN_ERR_UNSUPPORTED. Pixels are FP16 NCHW planes (1, C, H, W)
 * in host memory (uint16 bit patterns).
 */
#ifndef DENOISER_B200_IO_H
#define DENOISER_B200_IO_H

#include "denoiser_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Channels (as loaded), height and width of an image file. load_image /
 * load_exr (image_io.h:11, exr_io.h:11) decide the same numbers. */
int dn_image_probe(const char* path, int* channels, int* height, int* width);
/* Decode `path` into half_nchw (channels * height * width FP16 values); the
 * sizes must equal dn_image_probe's. */
int dn_image_read(const char* path, void* half_nchw, int channels, int height, int width);
/* Encode by extension (.png, .exr, .ppm/.pgm, .pfm); save_image / save_exr
 * (image_io.h:16, exr_io.h:16). */
int dn_image_write(const char* path, const void* half_nchw, int channels, int height, int width);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* DENOISER_B200_IO_H */
