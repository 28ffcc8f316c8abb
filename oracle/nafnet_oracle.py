"""CPU oracle for the NAFNet inference path (TEST INFRASTRUCTURE ONLY).

This file is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg (and its
``--impl reference`` arm) may import it. The engine never routes through it.

It restates, in plain PyTorch fp32 on the CPU, the forward passes of the
reference project ginzburg-dev/ml-video-denoiser:

* ``nafnet_forward``            training/models.py:542-577   (NAFNet.forward)
* ``nafblock``                  training/models.py:166-185   (NAFBlock.forward)
* ``layer_norm2d``              training/models.py:86-94     (LayerNorm2d.forward)
* ``pad_to_multiple``/``unpad`` training/models.py:42-62
* ``nafnet_temporal_forward``   training/models.py:738-808   (current PyTorch NAFNetTemporal)
* ``warp_grid``                 training/models.py:321-343   (_warp, grid_sample
                                align_corners=True, border padding)
* ``nafnet_temporal_legacy_forward``
                                src/models/nafnet_temporal.cu:363-503 (the C++ engine's
                                temporal design: temporal_mix(concat(ref, mean(nbrs))))
* ``warp_pixel``                src/kernels/nafnet_kernels.cu:212-262 (pixel offsets,
                                border clamp, ch0 = dx, ch1 = dy)
* ``deform_conv2d``             src/kernels/deform_im2col.cuh:34-142 + the GEMM of
                                src/layers/deform_conv2d.cu:134-182 (DCNv2, sigmoid mask)
* ``aligned_temporal_forward``  the temporal model with deformable alignment: feature
                                conv, offset/mask conv, DCN per neighbour, 1x1 fusion,
                                NAFNet trunk (no reference model wires the DCN; this
                                composition of the restatements is the checker for it)

Architecture is discovered from the weight keys the same way the C++ engine
does (src/models/nafnet.cu:78-92). Parameters are the fp32 values of the
fp16 ``.bin`` files (what the FP16 engine sees). The oracle is pinned against
golden vectors produced by running the reference's own PyTorch modules
(``tests/golden/make_golden.py``; checked by ``tests/test_oracle_golden.py``).
"""
from __future__ import annotations

import json
import os

import numpy as np
import torch
import torch.nn.functional as F

# ---------------------------------------------------------------------------
# Weights (reference format: training/export.py:48-118, src/weight_loader.cc:91-175)
# ---------------------------------------------------------------------------


def load_manifest(path: str) -> tuple[dict, dict]:
    """Return (params as fp32 torch tensors, architecture dict)."""
    with open(path) as f:
        man = json.load(f)
    base = os.path.dirname(path)
    params = {}
    for layer in man["layers"]:
        dt = np.float16 if layer["dtype"] == "float16" else np.float32
        arr = np.fromfile(os.path.join(base, layer["file"]), dtype=dt)
        params[layer["name"]] = torch.from_numpy(arr.astype(np.float32).reshape(layer["shape"]))
    return params, man.get("architecture", {})


def as_torch(params: dict) -> dict:
    return {k: (v if isinstance(v, torch.Tensor) else torch.from_numpy(np.asarray(v, np.float32)))
            for k, v in params.items()}


def count_levels(p: dict, root: str) -> int:
    n = 0
    while f"{root}.{n}.0.conv1.weight" in p:
        n += 1
    return n


def count_blocks(p: dict, root: str) -> int:
    n = 0
    while f"{root}.{n}.conv1.weight" in p:
        n += 1
    return n


# ---------------------------------------------------------------------------
# Building blocks
# ---------------------------------------------------------------------------


def pad_to_multiple(x: torch.Tensor, multiple: int):
    """Right/bottom reflect pad so H, W divide `multiple` (models.py:42-54)."""
    h, w = x.shape[-2:]
    ph = (multiple - h % multiple) % multiple
    pw = (multiple - w % multiple) % multiple
    return F.pad(x, (0, pw, 0, ph), mode="reflect"), (ph, pw)


def unpad(x: torch.Tensor, pad) -> torch.Tensor:
    ph, pw = pad
    h, w = x.shape[-2:]
    return x[..., : h - ph, : w - pw]


def layer_norm2d(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float = 1e-6):
    """LayerNorm over C at each pixel, then affine (models.py:86-94)."""
    mu = x.mean(dim=1, keepdim=True)
    var = ((x - mu) ** 2).mean(dim=1, keepdim=True)
    y = (x - mu) / torch.sqrt(var + eps)
    return y * w[None, :, None, None] + b[None, :, None, None]


def simple_gate(x: torch.Tensor) -> torch.Tensor:
    """x[:C] * x[C:] (models.py:106-108)."""
    a, b = x.chunk(2, dim=1)
    return a * b


def conv(p: dict, name: str, x: torch.Tensor, padding: int = 0, stride: int = 1,
         groups: int = 1, bias: bool = True) -> torch.Tensor:
    return F.conv2d(x, p[f"{name}.weight"], p.get(f"{name}.bias") if bias else None,
                    stride=stride, padding=padding, groups=groups)


def nafblock(p: dict, pre: str, x: torch.Tensor) -> torch.Tensor:
    """NAFBlock.forward (models.py:166-185)."""
    ident = x
    y = layer_norm2d(x, p[f"{pre}.norm1.weight"], p[f"{pre}.norm1.bias"])
    y = conv(p, f"{pre}.conv1", y)
    y = conv(p, f"{pre}.conv2", y, padding=1, groups=y.shape[1])
    y = simple_gate(y)
    s = conv(p, f"{pre}.sca.1", y.mean(dim=(2, 3), keepdim=True))
    y = conv(p, f"{pre}.conv3", y * s)
    x = ident + y * p[f"{pre}.beta"]
    ident = x
    y = layer_norm2d(x, p[f"{pre}.norm2.weight"], p[f"{pre}.norm2.bias"])
    y = conv(p, f"{pre}.conv4", y)
    y = simple_gate(y)
    y = conv(p, f"{pre}.conv5", y)
    return ident + y * p[f"{pre}.gamma"]


def stage(p: dict, root: str, x: torch.Tensor) -> torch.Tensor:
    for i in range(count_blocks(p, root)):
        x = nafblock(p, f"{root}.{i}", x)
    return x


def upsample(p: dict, lvl: int, x: torch.Tensor) -> torch.Tensor:
    """1x1 (no bias) + PixelShuffle(2) (models.py:217-224)."""
    return F.pixel_shuffle(F.conv2d(x, p[f"ups.{lvl}.body.0.weight"]), 2)


def match_spatial(a: torch.Tensor, b: torch.Tensor):
    """Crop both to the shared (H, W) (models.py:227-243)."""
    h = min(a.shape[-2], b.shape[-2])
    w = min(a.shape[-1], b.shape[-1])
    return a[..., :h, :w], b[..., :h, :w]


# ---------------------------------------------------------------------------
# NAFNet (spatial)
# ---------------------------------------------------------------------------


@torch.no_grad()
def nafnet_forward(p: dict, x: torch.Tensor) -> torch.Tensor:
    """NAFNet.forward (models.py:542-577). x: (B, C_in, H, W) fp32."""
    levels = count_levels(p, "encoders")
    x = torch.nan_to_num(x, nan=0.0, posinf=0.0, neginf=0.0)
    beauty = x[:, :3]
    x, pad = pad_to_multiple(x, 2 ** levels)
    x = conv(p, "intro", x, padding=1)
    skips = []
    for lvl in range(levels):
        x = stage(p, f"encoders.{lvl}", x)
        skips.append(x)
        x = conv(p, f"downs.{lvl}.body", x, stride=2)
    x = stage(p, "middle", x)
    for lvl in range(levels):
        x = upsample(p, lvl, x)
        x, s = match_spatial(x, skips[levels - 1 - lvl])
        x = stage(p, f"decoders.{lvl}", x + s)
    return beauty + unpad(conv(p, "ending", x, padding=1), pad)


# ---------------------------------------------------------------------------
# Temporal models
# ---------------------------------------------------------------------------


def warp_grid(feat: torch.Tensor, offset: torch.Tensor) -> torch.Tensor:
    """_warp (models.py:321-343): grid_sample, align_corners=True, border."""
    b, _, h, w = feat.shape
    gy, gx = torch.meshgrid(torch.linspace(-1.0, 1.0, h), torch.linspace(-1.0, 1.0, w),
                            indexing="ij")
    base = torch.stack([gx, gy], dim=-1).unsqueeze(0)
    norm = torch.stack([offset[:, 0] / (w / 2.0), offset[:, 1] / (h / 2.0)], dim=-1)
    return F.grid_sample(feat, base + norm, mode="bilinear", padding_mode="border",
                         align_corners=True)


def offset_head(p: dict, lvl: int, x: torch.Tensor) -> torch.Tensor:
    """DW3x3 -> PW1x1 -> ReLU -> PW1x1 (models.py:346-372)."""
    pre = f"offset_heads.{lvl}"
    y = F.conv2d(x, p[f"{pre}.0.weight"], padding=1, groups=x.shape[1])
    y = F.relu(F.conv2d(y, p[f"{pre}.1.weight"]))
    return F.conv2d(y, p[f"{pre}.3.weight"], p[f"{pre}.3.bias"])


def mix_stage(p: dict, root: str, x: torch.Tensor) -> torch.Tensor:
    """Conv1x1 (T*C -> C) followed by the NAFBlocks of ``root`` (models.py:693-698, 729-736)."""
    x = conv(p, f"{root}.0", x)
    i = 1
    while f"{root}.{i}.conv1.weight" in p:
        x = nafblock(p, f"{root}.{i}", x)
        i += 1
    return x


def encode_frames(p: dict, frames: torch.Tensor, levels: int):
    """Shared intro + encoders on a (B*T, C, H, W) batch: skips per level + deep features."""
    x = conv(p, "intro", frames, padding=1)
    skips = []
    for lvl in range(levels):
        x = stage(p, f"encoders.{lvl}", x)
        skips.append(x)
        x = conv(p, f"downs.{lvl}.body", x, stride=2)
    return skips, x


def decode(p: dict, x: torch.Tensor, fused_skips: list, levels: int) -> torch.Tensor:
    for lvl in range(levels):
        x = upsample(p, lvl, x)
        x, s = match_spatial(x, fused_skips[levels - 1 - lvl])
        x = stage(p, f"decoders.{lvl}", x + s)
    return conv(p, "ending", x, padding=1)


@torch.no_grad()
def nafnet_temporal_forward(p: dict, clip: torch.Tensor) -> torch.Tensor:
    """Current PyTorch NAFNetTemporal.forward (models.py:738-808). clip: (B, T, C, H, W)."""
    b, t, c, h, w = clip.shape
    levels = count_levels(p, "encoders")
    ref = t // 2
    clip = torch.nan_to_num(clip, nan=0.0, posinf=0.0, neginf=0.0)
    beauty = clip[:, ref, :3]
    padded = []
    for i in range(t):
        xp, pad = pad_to_multiple(clip[:, i], 2 ** levels)
        padded.append(xp)
    x = torch.stack(padded, dim=1).reshape(b * t, c, *padded[0].shape[-2:])
    skips, deep = encode_frames(p, x, levels)
    deep = deep.reshape(b, t, *deep.shape[1:])
    x = mix_stage(p, "bottleneck_mix", torch.cat([deep[:, i] for i in range(t)], dim=1))
    x = stage(p, "middle", x)
    use_warp = "offset_heads.0.0.weight" in p
    fused = []
    for lvl in range(levels):
        s = skips[lvl].reshape(b, t, *skips[lvl].shape[1:])
        feats = [s[:, i] for i in range(t)]
        if use_warp:
            rf = feats[ref]
            feats = [feats[i] if i == ref else
                     warp_grid(feats[i], offset_head(p, lvl, torch.cat([rf, feats[i]], dim=1)))
                     for i in range(t)]
        fused.append(mix_stage(p, f"temporal_mix.{lvl}", torch.cat(feats, dim=1)))
    return beauty + unpad(decode(p, x, fused, levels), pad)


def warp_pixel(feat: torch.Tensor, offset: torch.Tensor) -> torch.Tensor:
    """warp_bilinear_kernel (nafnet_kernels.cu:221-262): sample at (x+dx, y+dy) in
    pixel units, every tap clamped to the border; offset ch0 = dx, ch1 = dy."""
    n, c, h, w = feat.shape
    ys = torch.arange(h, dtype=torch.float32).view(1, h, 1)
    xs = torch.arange(w, dtype=torch.float32).view(1, 1, w)
    x = xs + offset[:, 0]
    y = ys + offset[:, 1]
    x0 = torch.floor(x)
    y0 = torch.floor(y)
    wx = (x - x0)[:, None]
    wy = (y - y0)[:, None]
    x0i = x0.long()
    y0i = y0.long()

    def tap(yi, xi):
        yi = yi.clamp(0, h - 1)
        xi = xi.clamp(0, w - 1)
        idx = (yi * w + xi).view(n, 1, h * w).expand(n, c, h * w)
        return torch.gather(feat.reshape(n, c, h * w), 2, idx).view(n, c, h, w)

    return (tap(y0i, x0i) * (1 - wy) * (1 - wx) + tap(y0i, x0i + 1) * (1 - wy) * wx
            + tap(y0i + 1, x0i) * wy * (1 - wx) + tap(y0i + 1, x0i + 1) * wy * wx)


@torch.no_grad()
def nafnet_temporal_legacy_forward(p: dict, clip: torch.Tensor, num_frames: int | None = None):
    """C++ NAFNetTemporal::forward (nafnet_temporal.cu:363-503): every frame through
    intro+encoders; middle on the reference frame's deep features only; per level
    skip = temporal_mix(concat(ref, mean_t(warp?(nbr_t)))), warp via offset_heads
    (a 1x1 conv on concat(ref, nbr)); decoder as the spatial model."""
    b, t, c, h, w = clip.shape
    levels = count_levels(p, "encoders")
    ref = t // 2
    beauty = clip[:, ref, :3]
    padded = []
    for i in range(t):
        xp, pad = pad_to_multiple(clip[:, i], 2 ** levels)
        padded.append(xp)
    x = torch.stack(padded, dim=1).reshape(b * t, c, *padded[0].shape[-2:])
    skips, deep = encode_frames(p, x, levels)
    deep = deep.reshape(b, t, *deep.shape[1:])
    x = stage(p, "middle", deep[:, ref])
    use_warp = "offset_heads.0.weight" in p
    fused = []
    for lvl in range(levels):
        s = skips[lvl].reshape(b, t, *skips[lvl].shape[1:])
        rf = s[:, ref]
        acc = torch.zeros_like(rf)
        for i in range(t):
            if i == ref:
                continue
            nb = s[:, i]
            if use_warp:
                off = conv(p, f"offset_heads.{lvl}", torch.cat([rf, nb], dim=1))
                nb = warp_pixel(nb, off)
            acc = acc + nb
        mean = acc / (t - 1)
        fused.append(conv(p, f"temporal_mix.{lvl}", torch.cat([rf, mean], dim=1)))
    return beauty + unpad(decode(p, x, fused, levels), pad)


# ---------------------------------------------------------------------------
# Deformable convolution (DCNv2)
# ---------------------------------------------------------------------------


def bilinear_zero(inp: torch.Tensor, hs: torch.Tensor, ws: torch.Tensor) -> torch.Tensor:
    """bilinear_sample (deform_im2col.cuh:34-69): zero outside; a point with
    h < -1, h > H, w < -1 or w > W samples to 0; out-of-range corners give 0.
    inp: (C, H, W); hs, ws: (C, *) sample coordinates per channel."""
    cdim, h, w = inp.shape
    outside = (hs < -1) | (hs > h) | (ws < -1) | (ws > w)
    h0 = torch.floor(hs)
    w0 = torch.floor(ws)
    dh = hs - h0
    dw = ws - w0
    h0 = h0.long()
    w0 = w0.long()
    flat = inp.reshape(cdim, h * w)

    def val(r, cc):
        ok = (r >= 0) & (r < h) & (cc >= 0) & (cc < w)
        idx = (r.clamp(0, h - 1) * w + cc.clamp(0, w - 1)).reshape(cdim, -1)
        return torch.gather(flat, 1, idx).reshape(r.shape) * ok

    v = (val(h0, w0) * (1 - dh) * (1 - dw) + val(h0, w0 + 1) * (1 - dh) * dw
         + val(h0 + 1, w0) * dh * (1 - dw) + val(h0 + 1, w0 + 1) * dh * dw)
    return torch.where(outside, torch.zeros_like(v), v)


@torch.no_grad()
def deform_conv2d(x: torch.Tensor, offsets: torch.Tensor, masks: torch.Tensor,
                  weight: torch.Tensor, bias: torch.Tensor | None, pad: int = 1,
                  stride: int = 1, dilation: int = 1, deform_groups: int = 8) -> torch.Tensor:
    """DeformConv2dLayer::forward (deform_conv2d.cu:105-184): im2col of
    bilinear(x, p + offset) * sigmoid(mask), then W @ col + bias.
    Offsets: channel 2*(g*kk + k) = dy, +1 = dx (deform_im2col.cuh:104-112)."""
    n, cin, h, w = x.shape
    cout, _, kh, kw = weight.shape
    ho = (h + 2 * pad - dilation * (kh - 1) - 1) // stride + 1
    wo = (w + 2 * pad - dilation * (kw - 1) - 1) // stride + 1
    kk = kh * kw
    cpg = cin // deform_groups
    out = torch.empty(n, cout, ho, wo)
    oy = torch.arange(ho, dtype=torch.float32).view(ho, 1) * stride - pad
    ox = torch.arange(wo, dtype=torch.float32).view(1, wo) * stride - pad
    for b in range(n):
        cols = torch.empty(cin, kk, ho * wo)
        for g in range(deform_groups):
            chans = slice(g * cpg, (g + 1) * cpg)
            for k in range(kk):
                ki, kj = divmod(k, kw)
                dy = offsets[b, 2 * (g * kk + k)]
                dx = offsets[b, 2 * (g * kk + k) + 1]
                m = torch.sigmoid(masks[b, g * kk + k])
                hs = (oy + ki * dilation + dy).reshape(1, -1).expand(cpg, -1)
                ws = (ox + kj * dilation + dx).reshape(1, -1).expand(cpg, -1)
                v = bilinear_zero(x[b, chans], hs, ws)
                cols[chans, k] = v * m.reshape(1, -1)
        res = weight.reshape(cout, cin * kk) @ cols.reshape(cin * kk, ho * wo)
        if bias is not None:
            res = res + bias.view(cout, 1)
        out[b] = res.view(cout, ho, wo)
    return out


def aligned_fusion(pa: dict, clip: torch.Tensor):
    """The alignment stage of the temporal NAFNet with deformable alignment,
    fp32: the trunk input fuse(concat(a_0 .. a_{T-1})) + frame_c, with
    a_t = DCN(f_t, offset(concat(f_c, f_t))) for t != c and a_c = f_c. The
    reference wires its DeformConv2dLayer (deform_conv2d.cu:105-184) into no
    model, so the wiring is this project's; its pieces are the restatements
    above. clip: (1, T, C, H, W); the centre frame is T // 2. Returns the
    fused image and the per-neighbour offsets/masks tensors (for statistics)."""
    t = clip.shape[1]
    c = t // 2
    feats = [conv(pa, "align.feat", clip[:, i], padding=1) for i in range(t)]
    n_off = pa["align.offset.weight"].shape[0] * 2 // 3
    dg = n_off // 18
    aligned, oms = [], []
    for i in range(t):
        if i == c:
            aligned.append(feats[c])
            continue
        om = conv(pa, "align.offset", torch.cat([feats[c], feats[i]], 1), padding=1)
        oms.append(om)
        aligned.append(deform_conv2d(feats[i], om[:, :n_off], om[:, n_off:], pa["align.dcn.weight"],
                                     pa["align.dcn.bias"], pad=1, deform_groups=dg))
    fused = conv(pa, "align.fuse", torch.cat(aligned, 1)) + clip[:, c]
    return fused, oms


def aligned_temporal_forward(pa: dict, pt: dict, clip: torch.Tensor):
    """Temporal NAFNet with deformable alignment, fp32: ``aligned_fusion``
    followed by the NAFNet trunk (``nafnet_forward``). Returns (1, 3, H, W)
    and the per-neighbour offsets/masks tensors."""
    fused, oms = aligned_fusion(pa, clip)
    return nafnet_forward(pt, fused), oms


# ---------------------------------------------------------------------------
# Metrics
# ---------------------------------------------------------------------------


def psnr(a: torch.Tensor, b: torch.Tensor, peak: float = 1.0) -> float:
    mse = float(((a.double() - b.double()) ** 2).mean())
    return float("inf") if mse == 0 else 10.0 * np.log10(peak * peak / mse)
