"""CPU oracle for the NCHW FP16 kernel launchers (TEST INFRASTRUCTURE ONLY).

This file is the checker, never the product: only ``tests/`` may import it.

Each function restates one ``denoiser::kernels::launch_*`` kernel of the
reference engine in numpy: FP16 inputs, FP32 arithmetic per element, one
round-to-nearest-even conversion to FP16 at the store, exactly as the CUDA
kernels do (``__half2float`` / ``__float2half``).

* ``reflect_pad``             src/kernels/model_kernels.cu:15-34
* ``crop``                    src/kernels/model_kernels.cu:40-56
* ``subtract_clamp``          src/kernels/model_kernels.cu:62-72
* ``concat_channels``         src/kernels/concat.cuh:19-41
* ``extract_frame``           src/kernels/nafnet_kernels.cu:16-33
* ``select_prefix_channels``  src/kernels/nafnet_kernels.cu:35-52
* ``layer_norm_affine``       src/kernels/nafnet_kernels.cu:54-92 (two-pass
                              mean / biased variance, eps 1e-6)
* ``simple_gate``             src/kernels/nafnet_kernels.cu:94-106 for N = 1;
                              for N > 1 the per-image channel split of
                              training/models.py:97-110 (SimpleGate.forward),
                              which the CUDA kernel's flat indexing only
                              matches at N = 1
* ``global_avg_pool``         src/kernels/nafnet_kernels.cu:108-126 (sequential
                              FP32 sum over the plane, then / (H*W))
* ``mul_channelwise``         src/kernels/nafnet_kernels.cu:128-141
* ``add``                     src/kernels/nafnet_kernels.cu:143-152
* ``mul_scalar``              src/kernels/nafnet_kernels.cu:154-163
* ``scaled_add``              src/kernels/nafnet_kernels.cu:165-180
* ``pixel_shuffle2x``         src/kernels/nafnet_kernels.cu:182-208
* ``warp_bilinear``           src/kernels/nafnet_kernels.cu:210-262
* ``upsample_bilinear``       src/layers/upsample.cu:10-45 (UpsampleLayer's
                              kernel: unclamped weights at the low border)

The restatements are pinned against torch's own CPU operators (F.pad
reflect, F.pixel_shuffle, channel LayerNorm, mean, grid arithmetic) in
``tests/test_kernels_oracle.py``: those are the operators the reference's
PyTorch model (training/models.py) uses for the same steps.
"""
from __future__ import annotations

import numpy as np

F16 = np.float16
F32 = np.float32


def _f(x):
    return np.asarray(x, dtype=F16).astype(F32)


def reflect_pad(x, H_out: int, W_out: int):
    """model_kernels.cu:29-33: h >= H_in -> 2*(H_in-1) - h (bottom/right only)."""
    x = np.asarray(x, dtype=F16)
    H_in, W_in = x.shape[-2:]
    hs = np.array([h if h < H_in else 2 * (H_in - 1) - h for h in range(H_out)])
    ws = np.array([w if w < W_in else 2 * (W_in - 1) - w for w in range(W_out)])
    return x[..., hs[:, None], ws[None, :]]


def crop(x, H_out: int, W_out: int):
    """model_kernels.cu:54-55: the top-left corner."""
    return np.ascontiguousarray(np.asarray(x, dtype=F16)[..., :H_out, :W_out])


def subtract_clamp(a, b):
    """model_kernels.cu:70-71: clamp(a - b, 0, 1), NaN passes through."""
    v = _f(a) - _f(b)
    v = np.where(v < 0, F32(0), np.where(v > 1, F32(1), v))
    return v.astype(F16)


def concat_channels(a, b):
    """concat.cuh:34-40."""
    return np.concatenate([np.asarray(a, dtype=F16), np.asarray(b, dtype=F16)], axis=1)


def extract_frame(clip, frame_idx: int):
    """nafnet_kernels.cu:30-32: clip (N,T,C,H,W) -> clip[:, frame_idx]."""
    return np.ascontiguousarray(np.asarray(clip, dtype=F16)[:, frame_idx])


def select_prefix_channels(x, C_out: int):
    """nafnet_kernels.cu:49-51."""
    return np.ascontiguousarray(np.asarray(x, dtype=F16)[:, :C_out])


def layer_norm_affine(x, weight, bias):
    """nafnet_kernels.cu:72-91: mean, then sum of squared deviations / C,
    inv_std = rsqrt(var + 1e-6), out = (x - mean) * inv_std * w + b."""
    v = _f(x)
    C = v.shape[1]
    mean = (v.sum(axis=1, keepdims=True, dtype=F32) / F32(C)).astype(F32)
    d = v - mean
    var = ((d * d).sum(axis=1, keepdims=True, dtype=F32) / F32(C)).astype(F32)
    inv_std = (F32(1) / np.sqrt(var + F32(1e-6))).astype(F32)
    w = np.asarray(weight).astype(F32).reshape(1, C, 1, 1)
    b = np.asarray(bias).astype(F32).reshape(1, C, 1, 1)
    return ((d * inv_std) * w + b).astype(F16)


def simple_gate(x):
    """Per image: out = x[:, :C] * x[:, C:] (nafnet_kernels.cu:103-105 at N = 1;
    training/models.py:106-110 for any N)."""
    v = _f(x)
    C = v.shape[1] // 2
    return (v[:, :C] * v[:, C:]).astype(F16)


def simple_gate_flat(x, N: int, C: int, H: int, W: int):
    """The CUDA kernel's literal indexing (nafnet_kernels.cu:101-105):
    output[i] = input[i] * input[i + C*H*W] over the flat buffer."""
    flat = _f(np.asarray(x).reshape(-1))
    n = N * C * H * W
    return (flat[:n] * flat[C * H * W:C * H * W + n]).astype(F16).reshape(N, C, H, W)


def global_avg_pool(x):
    """nafnet_kernels.cu:119-125: a sequential FP32 sum over each plane
    (np.cumsum accumulates in order), divided by H*W in FP32."""
    v = _f(x)
    N, C, H, W = v.shape
    flat = v.reshape(N * C, H * W)
    sums = np.cumsum(flat, axis=1, dtype=F32)[:, -1]
    return (sums / F32(H * W)).astype(F16).reshape(N, C)


def mul_channelwise(x, scale):
    """nafnet_kernels.cu:137-140: scale (N, C) FP16."""
    v = _f(x)
    s = _f(scale).reshape(v.shape[0], v.shape[1], 1, 1)
    return (v * s).astype(F16)


def add(a, b):
    """nafnet_kernels.cu:151."""
    return (_f(a) + _f(b)).astype(F16)


def mul_scalar(x, scalar: float):
    """nafnet_kernels.cu:162."""
    return (_f(x) * F32(scalar)).astype(F16)


def scaled_add(identity, residual, scale):
    """nafnet_kernels.cu:177-179: identity + residual * scale[c]."""
    v = _f(identity)
    s = np.asarray(scale).astype(F32).reshape(1, -1, 1, 1)
    return (v + _f(residual) * s).astype(F16)


def pixel_shuffle2x(x):
    """nafnet_kernels.cu:194-207: out[n, co, ho, wo] =
    in[n, 4*co + 2*(ho&1) + (wo&1), ho>>1, wo>>1]."""
    v = np.asarray(x, dtype=F16)
    N, C, H, W = v.shape
    return v.reshape(N, C // 4, 2, 2, H, W).transpose(0, 1, 4, 2, 5, 3).reshape(N, C // 4, 2 * H, 2 * W)


def warp_bilinear(feat, offset):
    """nafnet_kernels.cu:233-261: sample feat at (w + dx, h + dy) with
    border-clamped corners; offset channel 0 = dx, 1 = dy (pixels)."""
    f = _f(feat)
    o = _f(offset)
    N, C, H, W = f.shape
    hh, ww = np.meshgrid(np.arange(H, dtype=F32), np.arange(W, dtype=F32), indexing="ij")
    out = np.empty((N, C, H, W), dtype=F16)
    for n in range(N):
        x = ww + o[n, 0]
        y = hh + o[n, 1]
        fx0 = np.floor(x)
        fy0 = np.floor(y)
        wx = (x - fx0).astype(F32)
        wy = (y - fy0).astype(F32)
        x0 = fx0.astype(np.int64)
        y0 = fy0.astype(np.int64)
        xa, xb = np.clip(x0, 0, W - 1), np.clip(x0 + 1, 0, W - 1)
        ya, yb = np.clip(y0, 0, H - 1), np.clip(y0 + 1, 0, H - 1)
        fn = f[n]
        v00, v01 = fn[:, ya, xa], fn[:, ya, xb]
        v10, v11 = fn[:, yb, xa], fn[:, yb, xb]
        one = F32(1)
        val = (v00 * (one - wy) * (one - wx) + v01 * (one - wy) * wx + v10 * wy * (one - wx) + v11 * wy * wx)
        out[n] = val.astype(F16)
    return out


def upsample_bilinear(x, scale: int):
    """upsample.cu:24-44: src = (o + 0.5) / s - 0.5; low corner max(0, floor(src)),
    high corner min(low + 1, size - 1); weights from the unclamped src."""
    f = _f(x)
    N, C, H, W = f.shape
    ho = np.arange(H * scale, dtype=F32)
    wo = np.arange(W * scale, dtype=F32)
    hf = ((ho + F32(0.5)) / F32(scale) - F32(0.5)).astype(F32)
    wf = ((wo + F32(0.5)) / F32(scale) - F32(0.5)).astype(F32)
    h0 = np.maximum(0, np.floor(hf).astype(np.int64))
    w0 = np.maximum(0, np.floor(wf).astype(np.int64))
    h1 = np.minimum(h0 + 1, H - 1)
    w1 = np.minimum(w0 + 1, W - 1)
    dh = (hf - h0.astype(F32)).astype(F32)[:, None]
    dw = (wf - w0.astype(F32)).astype(F32)[None, :]
    one = F32(1)
    v00 = f[:, :, h0[:, None], w0[None, :]]
    v01 = f[:, :, h0[:, None], w1[None, :]]
    v10 = f[:, :, h1[:, None], w0[None, :]]
    v11 = f[:, :, h1[:, None], w1[None, :]]
    val = v00 * (one - dh) * (one - dw) + v01 * (one - dh) * dw + v10 * dh * (one - dw) + v11 * dh * dw
    return val.astype(F16)
