"""Frame-level inference over the engine, mirroring the reference's
training/infer.py:

* ``tile_inference``: overlapping tiles (overlap = tile_size // 8, stride =
  tile_size - overlap) blended with linear ramps, for frames too large to
  run at once (``_tile_inference`` :174-203, ``_tile_inference_temporal``
  :318-346, ``_make_ramp`` :206-216). As in the reference, the ramps start at
  0, so the outermost row and column of the frame get zero weight and come
  out as 0, and a tile narrower than the overlap is an error.
* ``denoise_temporal_sequence``: every frame of a sequence from its
  edge-replicated window, optionally averaged with the pass over the
  reversed sequence (``denoise_temporal_sequence`` :219-274).

The tile copies, the blending and the averaging are engine kernels
(include/denoiser_b200_infer.h); the model is any engine ``Model`` (or
``AlignedTemporal``) on FP16 CUDA tensors.
"""
from __future__ import annotations

import ctypes

from . import check, lib, stream_handle


def _p(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def tile_inference(model, x, tile_size: int, stream=None):
    """x: (1, C, H, W) for a spatial model or (1, T, C, H, W) for a temporal
    one, FP16 CUDA; returns the blended (1, 3, H, W) FP16 output."""
    import torch

    if tile_size <= 0:
        raise ValueError("tile_inference: tile_size must be positive")
    s = stream if stream is not None else torch.cuda.current_stream(x.device)
    sh = stream_handle(s)
    x = x.contiguous()
    h, w = x.shape[-2:]
    lead = tuple(x.shape[:-2])
    planes = 1
    for d in lead:
        planes *= d
    overlap = tile_size // 8
    stride = tile_size - overlap
    with torch.cuda.stream(s):
        acc = torch.zeros(3, h, w, dtype=torch.float32, device=x.device)
        wsum = torch.zeros(h, w, dtype=torch.float32, device=x.device)
        for y1 in range(0, h, stride):
            for x1 in range(0, w, stride):
                th, tw = min(y1 + tile_size, h) - y1, min(x1 + tile_size, w) - x1
                tile = torch.empty(lead + (th, tw), dtype=torch.float16, device=x.device)
                check(lib().dn_tile_extract(_p(x), _p(tile), planes, h, w, y1, x1, th, tw, sh))
                pred = model(tile, stream=s)
                check(lib().dn_tile_accumulate(_p(pred), ctypes.cast(acc.data_ptr(), ctypes.POINTER(ctypes.c_float)),
                                               ctypes.cast(wsum.data_ptr(), ctypes.POINTER(ctypes.c_float)), 3, h, w,
                                               y1, x1, th, tw, overlap, sh))
        out = torch.empty(1, 3, h, w, dtype=torch.float16, device=x.device)
        check(lib().dn_tile_normalize(ctypes.cast(acc.data_ptr(), ctypes.POINTER(ctypes.c_float)),
                                      ctypes.cast(wsum.data_ptr(), ctypes.POINTER(ctypes.c_float)), _p(out), 3, h, w,
                                      sh))
    return out


def _window(i: int, num_frames: int, n: int) -> list[int]:
    r = num_frames // 2
    return [min(max(i + t - r, 0), n - 1) for t in range(num_frames)]


def _sequence_pass(model, frames, num_frames: int, tile_size: int, stream):
    import torch

    n = len(frames)
    if tile_size > 0:
        outs = []
        for i in range(n):
            clip = torch.stack([frames[f] for f in _window(i, num_frames, n)], dim=0).unsqueeze(0)
            outs.append(tile_inference(model, clip, tile_size, stream)[0])
        return outs
    from . import sharding

    return [y for _, y in sharding.denoise_segment(model, lambda i: frames[i], n, 1, 0, num_frames=num_frames,
                                                    stream=stream)]


def denoise_temporal_sequence(model, frames, num_frames: int, temporal_flip: bool = True, tile_size: int = 0,
                              stream=None):
    """frames: list of (C, H, W) FP16 CUDA tensors of one size; returns the
    list of (3, H, W) FP16 outputs. With ``temporal_flip`` every output is
    the average of the forward pass and the pass over the reversed sequence."""
    import torch

    if not frames:
        return []
    if any(f.shape != frames[0].shape for f in frames):
        raise ValueError("Temporal inference requires all frames in a sequence to share shape")
    s = stream if stream is not None else torch.cuda.current_stream(frames[0].device)
    forward = _sequence_pass(model, frames, num_frames, tile_size, s)
    if not temporal_flip:
        return forward
    backward = _sequence_pass(model, frames[::-1], num_frames, tile_size, s)[::-1]
    out = []
    with torch.cuda.stream(s):
        for f, b in zip(forward, backward):
            y = torch.empty_like(f)
            check(lib().dn_average_pair(_p(f), _p(b), _p(y), f.numel(), stream_handle(s)))
            out.append(y)
    return out
