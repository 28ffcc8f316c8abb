"""ORACLE (test infrastructure only; nothing in the product imports it):
fp32 CPU restatement of the frame-level inference of the reference's
training/infer.py, with any model given as a callable on torch tensors.

* ``make_ramp``       — _make_ramp (infer.py:206-216)
* ``tile_inference``  — _tile_inference (:174-203) for (1, C, H, W) inputs and
                        _tile_inference_temporal (:318-346) for (1, T, C, H, W)
* ``denoise_temporal_sequence`` — denoise_temporal_sequence (:219-274) with
                        the edge-replicated windows of _clip_indices (:277-281)
Pinned by tests/golden/tile_*.npz and flip_*.npz, which
tests/golden/make_golden.py writes with the reference's own functions.
"""
from __future__ import annotations

import torch


def make_ramp(h: int, w: int, overlap: int) -> torch.Tensor:
    """(1, 1, h, w) blend weights: ones, the first `overlap` entries of each
    axis set to linspace(0, 1, overlap), then the last `overlap` to its
    reverse. Raises like the reference when an axis is shorter than overlap."""
    ry = torch.ones(h)
    rx = torch.ones(w)
    if overlap > 0:
        if overlap > h or overlap > w:
            raise RuntimeError(f"tile {h}x{w} narrower than the blend overlap {overlap}")
        ramp = torch.linspace(0.0, 1.0, overlap)
        ry[:overlap] = ramp
        ry[-overlap:] = ramp.flip(0)
        rx[:overlap] = ramp
        rx[-overlap:] = ramp.flip(0)
    return (ry[:, None] * rx[None, :])[None, None]


def tile_inference(model, x: torch.Tensor, tile_size: int) -> torch.Tensor:
    """Blend the model's outputs over overlapping tiles; (1, 3, H, W)."""
    h, w = x.shape[-2:]
    overlap = tile_size // 8
    stride = tile_size - overlap
    out = torch.zeros(1, 3, h, w)
    wsum = torch.zeros(1, 1, h, w)
    for y in range(0, h, stride):
        for xi in range(0, w, stride):
            y1, y2 = y, min(y + tile_size, h)
            x1, x2 = xi, min(xi + tile_size, w)
            pred = model(x[..., y1:y2, x1:x2].contiguous())
            ramp = make_ramp(pred.shape[-2], pred.shape[-1], overlap)
            out[:, :, y1:y2, x1:x2] += pred * ramp
            wsum[:, :, y1:y2, x1:x2] += ramp
    return out / wsum.clamp(min=1e-6)


def clip_indices(length: int, centre: int, num_frames: int) -> list[int]:
    r = num_frames // 2
    return [min(max(centre + o, 0), length - 1) for o in range(-r, r + 1)]


def denoise_temporal_sequence(model, frames: list, num_frames: int, temporal_flip: bool = True,
                              tile_size: int = 0) -> list:
    """frames: list of (C, H, W) float32 tensors; returns (3, H, W) outputs."""
    def one_pass(seq):
        outs = []
        for i in range(len(seq)):
            clip = torch.stack([seq[f] for f in clip_indices(len(seq), i, num_frames)])[None]
            y = tile_inference(model, clip, tile_size) if tile_size > 0 else model(clip)
            outs.append(y[0])
        return outs

    fwd = one_pass(frames)
    if not temporal_flip:
        return fwd
    bwd = one_pass(frames[::-1])[::-1]
    return [(f + b) * 0.5 for f, b in zip(fwd, bwd)]
