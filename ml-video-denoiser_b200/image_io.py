"""Image files as (1, C, H, W) FP16 numpy arrays through the engine's codecs
(include/denoiser_b200_io.h): PNG, EXR, PPM/PGM and PFM, with the pixel
semantics of the reference's load_image / save_image / load_exr / save_exr
(src/io/image_io.cc, src/io/exr_io.cc)."""
from __future__ import annotations

import ctypes

import numpy as np

from . import check, lib


def probe(path: str) -> tuple[int, int, int]:
    """(channels, height, width) the file loads as."""
    c, h, w = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    check(lib().dn_image_probe(str(path).encode(), ctypes.byref(c), ctypes.byref(h), ctypes.byref(w)))
    return c.value, h.value, w.value


def load(path: str) -> np.ndarray:
    """Decode an image file into a (1, C, H, W) float16 array."""
    c, h, w = probe(path)
    out = np.empty((1, c, h, w), dtype=np.float16)
    check(lib().dn_image_read(str(path).encode(), out.ctypes.data_as(ctypes.c_void_p), c, h, w))
    return out


def save(path: str, img) -> None:
    """Encode a (1, C, H, W) or (C, H, W) array by the file's extension."""
    a = np.ascontiguousarray(np.asarray(img, dtype=np.float16))
    if a.ndim == 4:
        if a.shape[0] != 1:
            raise ValueError("save: expected (1, C, H, W)")
        a = a[0]
    c, h, w = a.shape
    check(lib().dn_image_write(str(path).encode(), a.ctypes.data_as(ctypes.c_void_p), c, h, w))
