"""Synthetic weights, inputs and the manifest writer for the engine's workloads.

There is no network here and no trained checkpoint, so every workload runs
on seeded random-init weights and seeded synthetic frames:

* ``param_specs`` lists the parameter names and shapes of the reference's
  PyTorch models in ``state_dict`` order (``training/models.py``: NAFBlock
  :138-164, NAFDownsample :199-200, NAFUpsample :217-221, NAFNet :510-537,
  NAFNetTemporal :651-736, offset head :346-372) and of the reference C++
  engine's legacy temporal keys (``src/models/nafnet_temporal.cu:331-348``).
* ``init_params`` draws every tensor, including ``ending``, beta/gamma and
  the LayerNorm affine, so that no block is an identity (the reference's
  zero-init would make parity trivial).
* ``write_manifest`` writes the reference weight format: ``manifest.json``
  + ``weights/<name with . -> _>.bin``, raw little-endian C-contiguous
  (``training/export.py:48-118``).
* ``*_input`` build the seeded frames of the benchmark configurations.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass, field

import numpy as np


@dataclass
class NAFConfig:
    """Mirror of ``NAFNetConfig`` (``training/models.py:380-420``)."""

    in_channels: int = 3
    base_channels: int = 32
    enc_blocks: tuple = (1, 1, 1, 28)
    middle_blocks: int = 1
    dec_blocks: tuple = (1, 1, 1, 1)
    dw_expand: int = 1
    ffn_expand: int = 2

    @property
    def num_levels(self) -> int:
        return len(self.enc_blocks)


# Benchmark architectures.
# tiny w16: 4 levels of 1 block, 1 middle block, default expansions (1.47 M params).
CONFIG_TINY_W16 = NAFConfig(base_channels=16, enc_blocks=(1, 1, 1, 1), middle_blocks=1,
                            dec_blocks=(1, 1, 1, 1), dw_expand=1, ffn_expand=2)
# NAFNet-w32 in the paper's expansion convention (DW x2 and FFN x2 relative to
# C) is dw_expand=1 / ffn_expand=1 in the repo's convention (29.16 M params).
CONFIG_W32 = NAFConfig(base_channels=32, enc_blocks=(2, 2, 4, 8), middle_blocks=12,
                       dec_blocks=(2, 2, 2, 2), dw_expand=1, ffn_expand=1)
# Repo-literal reading of "expansion 2" (64.68 M params).
CONFIG_W32_LITERAL = NAFConfig(base_channels=32, enc_blocks=(2, 2, 4, 8), middle_blocks=12,
                               dec_blocks=(2, 2, 2, 2), dw_expand=2, ffn_expand=2)


# ---------------------------------------------------------------------------
# Parameter specs (state_dict order of the reference models)
# ---------------------------------------------------------------------------

def _block_specs(prefix: str, c: int, dw_expand: int, ffn_expand: int) -> list:
    dw = c * dw_expand
    ffn = c * ffn_expand
    return [
        (f"{prefix}.beta", (1, c, 1, 1)),
        (f"{prefix}.gamma", (1, c, 1, 1)),
        (f"{prefix}.norm1.weight", (c,)),
        (f"{prefix}.norm1.bias", (c,)),
        (f"{prefix}.conv1.weight", (2 * dw, c, 1, 1)),
        (f"{prefix}.conv1.bias", (2 * dw,)),
        (f"{prefix}.conv2.weight", (2 * dw, 1, 3, 3)),
        (f"{prefix}.conv2.bias", (2 * dw,)),
        (f"{prefix}.sca.1.weight", (dw, dw, 1, 1)),
        (f"{prefix}.sca.1.bias", (dw,)),
        (f"{prefix}.conv3.weight", (c, dw, 1, 1)),
        (f"{prefix}.conv3.bias", (c,)),
        (f"{prefix}.norm2.weight", (c,)),
        (f"{prefix}.norm2.bias", (c,)),
        (f"{prefix}.conv4.weight", (2 * ffn, c, 1, 1)),
        (f"{prefix}.conv4.bias", (2 * ffn,)),
        (f"{prefix}.conv5.weight", (c, ffn, 1, 1)),
        (f"{prefix}.conv5.bias", (c,)),
    ]


def param_specs(cfg: NAFConfig, temporal: str | None = None, num_frames: int = 3,
                use_warp: bool = False) -> list:
    """Ordered (name, shape) list.

    temporal: None (spatial NAFNet), "py" (current PyTorch NAFNetTemporal,
    ``training/models.py:651-736``) or "legacy" (keys read by the reference
    C++ NAFNetTemporal, ``src/models/nafnet_temporal.cu:331-348``).
    """
    b = cfg.base_channels
    ex = (cfg.dw_expand, cfg.ffn_expand)
    specs = [("intro.weight", (b, cfg.in_channels, 3, 3)), ("intro.bias", (b,))]
    if temporal is None:
        specs += [("ending.weight", (3, b, 3, 3)), ("ending.bias", (3,))]
    ch = b
    enc = []
    for lvl, nb in enumerate(cfg.enc_blocks):
        for i in range(nb):
            enc += _block_specs(f"encoders.{lvl}.{i}", ch, *ex)
        ch *= 2
    specs += enc
    ch = b
    downs = []
    enc_ch = []
    for lvl in range(cfg.num_levels):
        downs += [(f"downs.{lvl}.body.weight", (2 * ch, ch, 2, 2)),
                  (f"downs.{lvl}.body.bias", (2 * ch,))]
        enc_ch.append(ch)
        ch *= 2
    specs += downs
    if temporal == "py":
        specs += [("bottleneck_mix.0.weight", (ch, num_frames * ch, 1, 1)),
                  ("bottleneck_mix.0.bias", (ch,))]
        for i in (1, 2):
            specs += _block_specs(f"bottleneck_mix.{i}", ch, *ex)
    middle = []
    for i in range(cfg.middle_blocks):
        middle += _block_specs(f"middle.{i}", ch, *ex)
    ups = []
    dec = []
    for lvl, nb in enumerate(cfg.dec_blocks):
        ups.append((f"ups.{lvl}.body.0.weight", (2 * ch, ch, 1, 1)))
        ch //= 2
        for i in range(nb):
            dec += _block_specs(f"decoders.{lvl}.{i}", ch, *ex)
    if temporal is None:
        # NAFNet registers decoders, ups, then middle (models.py:524-537).
        specs += dec + ups + middle
    else:
        # NAFNetTemporal registers middle, ups, decoders (models.py:700-707).
        specs += middle + ups + dec
    if temporal is not None:
        specs += [("ending.weight", (3, b, 3, 3)), ("ending.bias", (3,))]
    if temporal == "py":
        if use_warp:
            for lvl, c in enumerate(enc_ch):
                specs += [(f"offset_heads.{lvl}.0.weight", (2 * c, 1, 3, 3)),
                          (f"offset_heads.{lvl}.1.weight", (c, 2 * c, 1, 1)),
                          (f"offset_heads.{lvl}.3.weight", (2, c, 1, 1)),
                          (f"offset_heads.{lvl}.3.bias", (2,))]
        for lvl, c in enumerate(enc_ch):
            specs += [(f"temporal_mix.{lvl}.0.weight", (c, num_frames * c, 1, 1)),
                      (f"temporal_mix.{lvl}.0.bias", (c,))]
            for i in (1, 2):
                specs += _block_specs(f"temporal_mix.{lvl}.{i}", c, *ex)
    elif temporal == "legacy":
        for lvl, c in enumerate(enc_ch):
            specs += [(f"temporal_mix.{lvl}.weight", (c, 2 * c, 1, 1)),
                      (f"temporal_mix.{lvl}.bias", (c,))]
        if use_warp:
            for lvl, c in enumerate(enc_ch):
                specs += [(f"offset_heads.{lvl}.weight", (2, 2 * c, 1, 1)),
                          (f"offset_heads.{lvl}.bias", (2,))]
    return specs


# ---------------------------------------------------------------------------
# Initialisation
# ---------------------------------------------------------------------------

@dataclass
class InitScale:
    """Spread of the non-conv parameters (conv weights/biases are always
    kaiming-uniform with bound 1/sqrt(fan_in), PyTorch's Conv2d default)."""

    beta_gamma: float = 0.5     # beta, gamma ~ U(-s, s)
    ln_weight: float = 0.2      # LN weight ~ 1 + U(-s, s)
    ln_bias: float = 0.1        # LN bias ~ U(-s, s)
    offset_scale: float = 1.0   # multiplier on offset-head output layers


def _fan_in(shape) -> int:
    return int(np.prod(shape[1:])) if len(shape) > 1 else 1


def init_params(specs: list, seed: int, scale: InitScale | None = None) -> dict:
    """Seeded draw of every tensor in ``specs`` (float32 numpy arrays)."""
    s = scale or InitScale()
    rng = np.random.default_rng(seed)
    weights = {n: shp for n, shp in specs}
    out = {}
    for name, shape in specs:
        if name.endswith(".beta") or name.endswith(".gamma"):
            a = rng.uniform(-s.beta_gamma, s.beta_gamma, size=shape)
        elif ".norm" in name and name.endswith(".weight"):
            a = 1.0 + rng.uniform(-s.ln_weight, s.ln_weight, size=shape)
        elif ".norm" in name and name.endswith(".bias"):
            a = rng.uniform(-s.ln_bias, s.ln_bias, size=shape)
        elif name.endswith(".weight"):
            bound = 1.0 / math.sqrt(_fan_in(shape))
            a = rng.uniform(-bound, bound, size=shape)
        elif name.endswith(".bias"):
            wshape = weights.get(name[: -len(".bias")] + ".weight")
            bound = 1.0 / math.sqrt(_fan_in(wshape)) if wshape else 0.1
            a = rng.uniform(-bound, bound, size=shape)
        else:
            raise ValueError(f"no init rule for {name}")
        if name.startswith("offset_heads.") and (name.endswith(".3.weight") or name.endswith(".3.bias")
                                                  or name.count(".") == 2):
            a = a * s.offset_scale
        out[name] = a.astype(np.float32)
    return out


def round_fp16(params: dict) -> dict:
    """The weights the FP16 engine sees (export rounds every tensor to fp16)."""
    return {k: v.astype(np.float16).astype(np.float32) for k, v in params.items()}


# ---------------------------------------------------------------------------
# Manifest writer (reference weight format)
# ---------------------------------------------------------------------------

def write_manifest(out_dir: str, params: dict, arch: dict, dtype: str = "float16",
                   order: list | None = None) -> str:
    """Write ``manifest.json`` + ``weights/*.bin`` like ``training/export.py:48-118``."""
    wdir = os.path.join(out_dir, "weights")
    os.makedirs(wdir, exist_ok=True)
    np_dtype = np.float16 if dtype == "float16" else np.float32
    layers = []
    for name in (order or list(params.keys())):
        arr = np.ascontiguousarray(params[name].astype(np_dtype))
        fname = name.replace(".", "_") + ".bin"
        arr.tofile(os.path.join(wdir, fname))
        layers.append({"name": name, "shape": list(arr.shape), "dtype": dtype,
                       "file": f"weights/{fname}"})
    manifest = {"version": "1.0", "dtype": dtype, "architecture": arch, "layers": layers}
    path = os.path.join(out_dir, "manifest.json")
    with open(path, "w") as f:
        json.dump(manifest, f, indent=2)
    return path


def arch_block(cfg: NAFConfig, temporal: str | None = None, num_frames: int = 3,
               use_warp: bool = False) -> dict:
    """The ``architecture`` block of ``training/export.py:121-134``."""
    a = {"type": "nafnet_temporal" if temporal else "nafnet_residual",
         "base_channels": cfg.base_channels, "num_levels": cfg.num_levels,
         "in_channels": cfg.in_channels}
    if temporal:
        a["num_frames"] = num_frames
        a["use_warp"] = use_warp
    return a


def make_model_dir(out_dir: str, cfg: NAFConfig, seed: int, temporal: str | None = None,
                   num_frames: int = 3, use_warp: bool = False,
                   scale: InitScale | None = None) -> tuple[str, dict]:
    """Generate seeded weights, write them, return (manifest path, fp16-rounded params)."""
    specs = param_specs(cfg, temporal, num_frames, use_warp)
    params = init_params(specs, seed, scale)
    path = write_manifest(out_dir, params, arch_block(cfg, temporal, num_frames, use_warp),
                          order=[n for n, _ in specs])
    return path, round_fp16(params)


# ---------------------------------------------------------------------------
# Deformable-alignment front end of the temporal model with DCN alignment
# ---------------------------------------------------------------------------

ALIGN_FEAT = 64     # feature channels the DCN aligns
ALIGN_DG = 8        # deformable groups
# Gains on the kaiming-uniform draw of align.offset: the offset rows then give
# offsets of about N(0, 2 px) on the synthetic windows (feature RMS ~0.33),
# the mask rows raw masks of std ~1 (sigmoid spread over ~0.3-0.7).
ALIGN_OFFSET_GAIN = 10.0
ALIGN_MASK_GAIN = 5.0


def align_param_specs(num_frames: int = 5, feat: int = ALIGN_FEAT, dg: int = ALIGN_DG,
                      in_channels: int = 3) -> list:
    """Keys of the alignment front end (``aligned.AlignedTemporal``):
    feature conv 3x3 in->F, offset/mask conv 3x3 2F->3*dg*9 (2*dg*9 offsets
    [dy, dx] per (group, tap), then dg*9 raw masks), DCNv2 3x3 F->F, fusion
    1x1 T*F->in."""
    kk = 9
    return [("align.feat.weight", (feat, in_channels, 3, 3)), ("align.feat.bias", (feat,)),
            ("align.offset.weight", (3 * dg * kk, 2 * feat, 3, 3)), ("align.offset.bias", (3 * dg * kk,)),
            ("align.dcn.weight", (feat, feat, 3, 3)), ("align.dcn.bias", (feat,)),
            ("align.fuse.weight", (in_channels, num_frames * feat, 1, 1)), ("align.fuse.bias", (in_channels,))]


def make_align_dir(out_dir: str, seed: int, num_frames: int = 5, feat: int = ALIGN_FEAT, dg: int = ALIGN_DG,
                   in_channels: int = 3) -> tuple[str, dict]:
    """Seeded alignment weights in the reference format; returns (manifest path,
    fp16-rounded params)."""
    specs = align_param_specs(num_frames, feat, dg, in_channels)
    params = init_params(specs, seed)
    n_off = 2 * dg * 9
    for key in ("align.offset.weight", "align.offset.bias"):
        params[key][:n_off] *= ALIGN_OFFSET_GAIN
        params[key][n_off:] *= ALIGN_MASK_GAIN
    arch = {"type": "dcn_align", "in_channels": in_channels, "num_frames": num_frames,
            "feat_channels": feat, "deform_groups": dg}
    path = write_manifest(out_dir, params, arch, order=[n for n, _ in specs])
    return path, round_fp16(params)


# ---------------------------------------------------------------------------
# Synthetic frames
# ---------------------------------------------------------------------------

def gradient_sinusoid_input(h: int, w: int, seed: int, sigma: float = 25.0 / 255.0,
                            channels: int = 3) -> np.ndarray:
    """Tiny-config frame: gradient + sinusoid (period 16-64 px) + N(0, sigma), clamped.

    Shapes follow the reference's sample-image generator
    (``tests/gen_sample_images.py:30-56, 88-97``). Returns (1, C, h, w) float32.
    """
    rng = np.random.default_rng(seed)
    yy, xx = np.meshgrid(np.linspace(0, 1, h, dtype=np.float32),
                         np.linspace(0, 1, w, dtype=np.float32), indexing="ij")
    img = np.empty((channels, h, w), np.float32)
    for c in range(channels):
        gx, gy = rng.uniform(-0.5, 0.5, 2)
        period = rng.uniform(16, 64)
        theta = rng.uniform(0, np.pi)
        phase = rng.uniform(0, 2 * np.pi)
        u = (np.cos(theta) * xx * w + np.sin(theta) * yy * h) / period
        img[c] = 0.5 + gx * (xx - 0.5) + gy * (yy - 0.5) + 0.2 * np.sin(2 * np.pi * u + phase)
    img = img + rng.normal(0.0, sigma, img.shape).astype(np.float32)
    return np.clip(img, 0.0, 1.0)[None]


def smooth_noise(h: int, w: int, seed: int, channels: int = 3, octaves: int = 4) -> np.ndarray:
    """Seeded smooth value noise in [0, 1] (Perlin-style octaves), (C, h, w)."""
    rng = np.random.default_rng(seed)
    out = np.zeros((channels, h, w), np.float32)
    amp_total = 0.0
    for o in range(octaves):
        cells = 4 * (2 ** o)
        gh, gw = cells + 2, int(cells * w / max(h, 1)) + 2
        grid = rng.random((channels, gh, gw)).astype(np.float32)
        ys = np.linspace(0, cells, h, dtype=np.float32)
        xs = np.linspace(0, gw - 2, w, dtype=np.float32)
        y0 = np.floor(ys).astype(int)
        x0 = np.floor(xs).astype(int)
        fy = ys - y0
        fx = xs - x0
        fy = fy * fy * (3 - 2 * fy)
        fx = fx * fx * (3 - 2 * fx)
        # Separable: interpolate every grid row along x first (gh rows), then
        # pick the two rows of each output row (the same products and sums
        # as the four-corner form, in the same order).
        gx = grid[:, :, x0] * (1 - fx) + grid[:, :, x0 + 1] * fx
        top = gx[:, y0]
        bot = gx[:, y0 + 1]
        amp = 0.5 ** o
        out += amp * (top * (1 - fy[:, None]) + bot * fy[:, None])
        amp_total += amp
    out /= amp_total
    lo = out.min(axis=(1, 2), keepdims=True)
    hi = out.max(axis=(1, 2), keepdims=True)
    return (out - lo) / np.maximum(hi - lo, 1e-6)


def poisson_gaussian(clean: np.ndarray, seed: int, gain: float = 0.01,
                     read_sigma: float = 0.02) -> np.ndarray:
    """Poisson(clean/gain)*gain + N(0, read_sigma^2)
    (the formula of ``training/noise_generators.py:176-187``)."""
    rng = np.random.default_rng(seed)
    shot = rng.poisson(np.clip(clean, 0, None) / gain).astype(np.float32) * gain
    return shot + rng.normal(0.0, read_sigma, clean.shape).astype(np.float32)


def w32_frame(h: int = 1080, w: int = 1920, seed: int = 1) -> np.ndarray:
    """1080p frame: smooth noise + Poisson-Gaussian (gain 0.01, read 0.02), (1,3,h,w)."""
    clean = smooth_noise(h, w, seed)
    return poisson_gaussian(clean, seed + 1000)[None]


def temporal_window(t: int, h: int, w: int, seed: int, sigma: float = 20.0 / 255.0,
                    max_shift: int = 4) -> np.ndarray:
    """T frames of one smooth base translated by per-frame integer shifts in
    [-max_shift, max_shift], each with independent N(0, sigma). (1, T, 3, h, w)."""
    rng = np.random.default_rng(seed)
    m = max_shift
    base = smooth_noise(h + 2 * m, w + 2 * m, seed)
    frames = []
    for _ in range(t):
        dy, dx = rng.integers(-m, m + 1, 2)
        f = base[:, m + dy: m + dy + h, m + dx: m + dx + w]
        frames.append(f + rng.normal(0.0, sigma, f.shape).astype(np.float32))
    return np.stack(frames)[None].astype(np.float32)


def pan_clip_base(h: int, w: int, n_frames: int, seed: int, device="cuda"):
    """Smooth base image for a clip panned 1 px per frame, (3, h, w + n_frames)
    float32 on `device`: ``smooth_noise`` with the same seeded grids,
    evaluated with torch on the device (4K bases in milliseconds)."""
    import torch

    w = w + n_frames
    rng = np.random.default_rng(seed)
    out = torch.zeros((3, h, w), dtype=torch.float32, device=device)
    amp_total = 0.0
    for o in range(4):
        cells = 4 * (2 ** o)
        gh, gw = cells + 2, int(cells * w / max(h, 1)) + 2
        grid = torch.from_numpy(rng.random((3, gh, gw)).astype(np.float32)).to(device)
        ys = torch.linspace(0, cells, h, dtype=torch.float32, device=device)
        xs = torch.linspace(0, gw - 2, w, dtype=torch.float32, device=device)
        y0, x0 = ys.floor().long(), xs.floor().long()
        fy, fx = ys - y0, xs - x0
        fy = fy * fy * (3 - 2 * fy)
        fx = fx * fx * (3 - 2 * fx)
        gx = grid[:, :, x0] * (1 - fx) + grid[:, :, x0 + 1] * fx
        amp = 0.5 ** o
        out += amp * (gx[:, y0] * (1 - fy[:, None]) + gx[:, y0 + 1] * fy[:, None])
        amp_total += amp
    out /= amp_total
    lo = out.amin(dim=(1, 2), keepdim=True)
    hi = out.amax(dim=(1, 2), keepdim=True)
    return (out - lo) / (hi - lo).clamp_min(1e-6)


def pan_clip_frame(base, i: int, w: int, seed: int, gain: float = 0.01, read_sigma: float = 0.02):
    """Frame i of the panned clip as a (1, 3, h, w) FP16 torch tensor on the
    device of `base` (a float32 torch tensor from ``pan_clip_base``): the
    window base[:, :, i:i+w] with Poisson-Gaussian noise (the formula of
    ``training/noise_generators.py:176-187``), drawn from a generator seeded
    with (seed, i) on that device."""
    import torch

    g = torch.Generator(device=base.device)
    g.manual_seed(int(seed) * 1000003 + int(i))
    clean = base[:, :, i:i + w].clamp_min(0.0)
    shot = torch.poisson(clean / gain, generator=g) * gain
    noisy = shot + torch.randn(clean.shape, generator=g, device=base.device) * read_sigma
    return noisy.half().unsqueeze(0).contiguous()
