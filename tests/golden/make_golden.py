"""Generate the golden vectors that pin the oracle to the reference.

Run in a container that has the reference checkout (read-only):

    python tests/golden/make_golden.py --reference /root/reference/training

It imports the reference's own PyTorch modules (``training/models.py``),
loads the engine's seeded synthetic weights into them (after checking that
the parameter names, shapes and order of ``synth.param_specs`` equal the
reference ``state_dict``), runs them in fp32 on the CPU and writes
``tests/golden/<case>.npz`` with the input and the expected output. The
weights themselves are not stored: they are regenerated from (config, seed)
by ``synth.init_params``.

Cases:
* spatial NAFNet (``NAFNet.forward``, models.py:542-577) at aligned,
  ragged and multi-channel shapes;
* current PyTorch NAFNetTemporal (models.py:738-808), with and without the
  warp heads;
* the C++ engine's legacy temporal wiring (nafnet_temporal.cu:363-503),
  assembled here from the reference's own NAFNet modules (its temporal_mix /
  offset heads are plain 1x1 convs) and a pixel-unit warp that follows
  ``warp_bilinear_kernel`` (nafnet_kernels.cu:221-262);
* frame-level inference of training/infer.py run by its own functions:
  ``_tile_inference`` (tiled spatial, ramp blending) and
  ``denoise_temporal_sequence`` with temporal flip averaging (untiled and
  tiled);
* DCNv2 (deform_im2col.cuh + deform_conv2d.cu) through the third-party
  ``torchvision.ops.deform_conv2d`` (torchvision 0.26.0) with
  mask = sigmoid(raw mask) and the same [dy, dx] offset layout.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from __graft_entry__ import load_package  # noqa: E402

synth = __import__(load_package().__name__ + ".synth", fromlist=["synth"])

# name -> (config kwargs, model kind, seeds, input spec)
CASES = {
    "spatial_w16l4_64x64": dict(cfg=dict(base_channels=16, enc_blocks=(1, 1, 1, 1), middle_blocks=1,
                                         dec_blocks=(1, 1, 1, 1), dw_expand=1, ffn_expand=2),
                                kind="spatial", wseed=0, shape=(1, 3, 64, 64), xseed=10),
    "spatial_w16l4_37x53": dict(cfg=dict(base_channels=16, enc_blocks=(1, 1, 1, 1), middle_blocks=1,
                                         dec_blocks=(1, 1, 1, 1), dw_expand=1, ffn_expand=2),
                                kind="spatial", wseed=0, shape=(1, 3, 37, 53), xseed=11),
    "spatial_w32dw1_48x40": dict(cfg=dict(base_channels=32, enc_blocks=(2, 1, 1), middle_blocks=2,
                                          dec_blocks=(1, 2, 1), dw_expand=1, ffn_expand=1),
                                 kind="spatial", wseed=1, shape=(1, 3, 48, 40), xseed=12),
    "spatial_w8_9ch_dw2_30x44": dict(cfg=dict(in_channels=9, base_channels=8, enc_blocks=(1, 2, 1),
                                              middle_blocks=2, dec_blocks=(1, 1, 1), dw_expand=2,
                                              ffn_expand=1),
                                     kind="spatial", wseed=3, shape=(2, 9, 30, 44), xseed=13),
    "temporal_py_w8l2_t3_warp": dict(cfg=dict(base_channels=8, enc_blocks=(1, 1), middle_blocks=1,
                                              dec_blocks=(1, 1), dw_expand=1, ffn_expand=1),
                                     kind="temporal_py", frames=3, warp=True, wseed=4,
                                     shape=(1, 3, 3, 28, 36), xseed=14),
    "temporal_py_w8l2_t5": dict(cfg=dict(base_channels=8, enc_blocks=(1, 1), middle_blocks=1,
                                         dec_blocks=(1, 1), dw_expand=1, ffn_expand=2),
                                kind="temporal_py", frames=5, warp=False, wseed=5,
                                shape=(1, 5, 3, 32, 32), xseed=15),
    "temporal_legacy_w8l2_t3_warp": dict(cfg=dict(base_channels=8, enc_blocks=(1, 1), middle_blocks=1,
                                                  dec_blocks=(1, 1), dw_expand=1, ffn_expand=1),
                                         kind="temporal_legacy", frames=3, warp=True, wseed=6,
                                         shape=(1, 3, 3, 24, 40), xseed=16),
    "temporal_legacy_w8l2_t5": dict(cfg=dict(base_channels=8, enc_blocks=(1, 1), middle_blocks=1,
                                             dec_blocks=(1, 1), dw_expand=1, ffn_expand=2),
                                    kind="temporal_legacy", frames=5, warp=False, wseed=7,
                                    shape=(1, 5, 3, 32, 32), xseed=17),
    "dcn_c16_dg4_20x24": dict(kind="dcn", cin=16, cout=16, dg=4, hw=(20, 24), seed=8),
}

# Frame-level inference (training/infer.py) through the reference's own
# functions: tiled spatial inference, and temporal sequences with flip
# averaging (untiled and tiled).
CASES.update({
    "tile_spatial_w16_70x90_t32": dict(cfg=dict(base_channels=16, enc_blocks=(1, 1), middle_blocks=1,
                                                dec_blocks=(1, 1), dw_expand=1, ffn_expand=2),
                                       kind="tile_spatial", wseed=6, shape=(1, 3, 70, 90), xseed=16, tile=32),
    "flip_temporal_py_w8_t3_seq5": dict(cfg=dict(base_channels=8, enc_blocks=(1, 1), middle_blocks=1,
                                                 dec_blocks=(1, 1), dw_expand=1, ffn_expand=1),
                                        kind="flip_temporal", frames=3, warp=False, wseed=7,
                                        shape=(5, 3, 24, 40), xseed=17, tile=0),
    "flip_temporal_py_w8_t3_seq4_t16": dict(cfg=dict(base_channels=8, enc_blocks=(1, 1), middle_blocks=1,
                                                     dec_blocks=(1, 1), dw_expand=1, ffn_expand=1),
                                            kind="flip_temporal", frames=3, warp=True, wseed=8,
                                            shape=(4, 3, 24, 40), xseed=18, tile=16),
})

TEMPORAL_KIND = {"spatial": None, "temporal_py": "py", "temporal_legacy": "legacy", "tile_spatial": None,
                 "flip_temporal": "py"}


def make_input(spec: dict) -> np.ndarray:
    shape = spec["shape"]
    rng = np.random.default_rng(spec["xseed"])
    x = rng.uniform(0.0, 1.0, size=shape).astype(np.float32)
    if len(shape) == 4 and shape[1] == 3:
        x = synth.gradient_sinusoid_input(shape[2], shape[3], spec["xseed"])
        x = np.repeat(x, shape[0], axis=0)
    return x.astype(np.float16).astype(np.float32)


def load_into(model: torch.nn.Module, params: dict) -> None:
    sd = model.state_dict()
    ours = list(params.keys())
    theirs = list(sd.keys())
    if ours != theirs:
        raise SystemExit(f"parameter names/order differ:\n ours  {ours[:8]}...\n theirs {theirs[:8]}...")
    for k in theirs:
        if tuple(sd[k].shape) != tuple(params[k].shape):
            raise SystemExit(f"shape mismatch for {k}: {tuple(sd[k].shape)} vs {params[k].shape}")
    model.load_state_dict({k: torch.from_numpy(v) for k, v in params.items()})
    model.eval()


def warp_pixel_ref(feat: torch.Tensor, off: torch.Tensor) -> torch.Tensor:
    """Per-element restatement of warp_bilinear_kernel (nafnet_kernels.cu:221-262)."""
    n, c, h, w = feat.shape
    out = torch.empty_like(feat)
    f = feat.numpy()
    o = off.numpy()
    res = out.numpy()
    for b in range(n):
        for y in range(h):
            for x in range(w):
                fx = x + float(o[b, 0, y, x])
                fy = y + float(o[b, 1, y, x])
                x0 = int(np.floor(fx))
                y0 = int(np.floor(fy))
                wx = fx - x0
                wy = fy - y0

                def s(yy, xx):
                    return f[b, :, min(max(yy, 0), h - 1), min(max(xx, 0), w - 1)]

                res[b, :, y, x] = (s(y0, x0) * (1 - wy) * (1 - wx) + s(y0, x0 + 1) * (1 - wy) * wx
                                   + s(y0 + 1, x0) * wy * (1 - wx) + s(y0 + 1, x0 + 1) * wy * wx)
    return out


def legacy_forward(m, p: dict, clip: torch.Tensor, levels: int) -> torch.Tensor:
    """C++ NAFNetTemporal wiring with the reference's NAFNet modules (m)."""
    from models import _match_spatial_size, _pad_to_multiple, _unpad

    b, t, c, h, w = clip.shape
    ref = t // 2
    beauty = clip[:, ref, :3]
    feats, pad = [], None
    for i in range(t):
        xp, pad = _pad_to_multiple(clip[:, i], 2 ** levels)
        feats.append(xp)
    skips_t, deep_t = [], []
    for i in range(t):
        x = m.intro(feats[i])
        sk = []
        for enc, down in zip(m.encoders, m.downs):
            x = enc(x)
            sk.append(x)
            x = down(x)
        skips_t.append(sk)
        deep_t.append(x)
    x = m.middle(deep_t[ref])
    fused = []
    for lvl in range(levels):
        rf = skips_t[ref][lvl]
        acc = torch.zeros_like(rf)
        for i in range(t):
            if i == ref:
                continue
            nb = skips_t[i][lvl]
            if f"offset_heads.{lvl}.weight" in p:
                off = F.conv2d(torch.cat([rf, nb], 1), torch.from_numpy(p[f"offset_heads.{lvl}.weight"]),
                               torch.from_numpy(p[f"offset_heads.{lvl}.bias"]))
                nb = warp_pixel_ref(nb, off)
            acc = acc + nb
        mean = acc / (t - 1)
        fused.append(F.conv2d(torch.cat([rf, mean], 1), torch.from_numpy(p[f"temporal_mix.{lvl}.weight"]),
                              torch.from_numpy(p[f"temporal_mix.{lvl}.bias"])))
    for lvl, (dec, up) in enumerate(zip(m.decoders, m.ups)):
        x = up(x)
        x, s = _match_spatial_size(x, fused[levels - 1 - lvl])
        x = dec(x + s)
    return beauty + _unpad(m.ending(x), (0, pad[1], 0, pad[3]))


def run_case(name: str, spec: dict):
    from models import NAFNet, NAFNetConfig, NAFNetTemporal

    if spec["kind"] == "dcn":
        import torchvision

        rng = np.random.default_rng(spec["seed"])
        cin, cout, dg = spec["cin"], spec["cout"], spec["dg"]
        h, w = spec["hw"]
        q = lambda a: a.astype(np.float16).astype(np.float32)  # noqa: E731
        x = q(rng.uniform(-1, 1, (1, cin, h, w)).astype(np.float32))
        off = rng.normal(0, 2.0, (1, 2 * dg * 9, h, w)).astype(np.float32)
        off = q(np.where(np.abs(off - np.round(off)) < 0.02, off + 0.05, off))
        mraw = q(rng.normal(0, 1.5, (1, dg * 9, h, w)).astype(np.float32))
        bound = 1.0 / np.sqrt(cin * 9)
        wt = q(rng.uniform(-bound, bound, (cout, cin, 3, 3)).astype(np.float32))
        bs = q(rng.uniform(-bound, bound, (cout,)).astype(np.float32))
        y = torchvision.ops.deform_conv2d(torch.from_numpy(x), torch.from_numpy(off), torch.from_numpy(wt),
                                          torch.from_numpy(bs), padding=1,
                                          mask=torch.sigmoid(torch.from_numpy(mraw)))
        return dict(x=x, offsets=off, masks=mraw, weight=wt, bias=bs, expected=y.numpy(),
                    meta=json.dumps(dict(kind="dcn", dg=dg, pad=1, stride=1, dilation=1)))

    cfg = synth.NAFConfig(**spec["cfg"])
    tk = TEMPORAL_KIND[spec["kind"]]
    frames = spec.get("frames", 3)
    warp = spec.get("warp", False)
    specs = synth.param_specs(cfg, tk, frames, warp)
    params = synth.round_fp16(synth.init_params(specs, spec["wseed"]))
    rcfg = NAFNetConfig(**{k: (tuple(v) if isinstance(v, (list, tuple)) else v) for k, v in spec["cfg"].items()})
    x = make_input(spec)
    if spec["kind"] in ("tile_spatial", "flip_temporal"):
        import infer as ref_infer  # the reference's training/infer.py

        dev = torch.device("cpu")
        with torch.no_grad():
            if spec["kind"] == "tile_spatial":
                m = NAFNet(rcfg)
                load_into(m, params)
                y = ref_infer._tile_inference(m.eval(), torch.from_numpy(x), spec["tile"], False, dev)
            else:
                m = NAFNetTemporal(rcfg, num_frames=frames, use_warp=warp)
                load_into(m, params)
                seq = [f.transpose(1, 2, 0).copy() for f in x]  # (H, W, C) frames
                outs = ref_infer.denoise_temporal_sequence(m.eval(), seq, dev, use_amp=False,
                                                          temporal_flip=True, tile_size=spec["tile"])
                y = torch.from_numpy(np.stack([o.transpose(2, 0, 1) for o in outs]))
        meta = dict(kind=spec["kind"], cfg=spec["cfg"], wseed=spec["wseed"], frames=frames, warp=warp,
                    tile=spec["tile"])
        return dict(x=x, expected=y.numpy().astype(np.float32), meta=json.dumps(meta))
    with torch.no_grad():
        if tk is None:
            m = NAFNet(rcfg)
            load_into(m, params)
            y = m(torch.from_numpy(x))
        elif tk == "py":
            m = NAFNetTemporal(rcfg, num_frames=frames, use_warp=warp)
            load_into(m, params)
            y = m(torch.from_numpy(x))
        else:
            m = NAFNet(rcfg)
            spatial = {k: v for k, v in params.items()
                       if not k.startswith(("temporal_mix", "offset_heads"))}
            load_into(m, {k: spatial[k] for k in m.state_dict().keys()})
            y = legacy_forward(m, params, torch.from_numpy(x), cfg.num_levels)
    meta = dict(kind=spec["kind"], cfg=spec["cfg"], wseed=spec["wseed"], frames=frames, warp=warp)
    return dict(x=x, expected=y.numpy().astype(np.float32), meta=json.dumps(meta))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="directory holding the reference's models.py (its training/ folder)")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    torch.manual_seed(0)
    for name, spec in CASES.items():
        if args.only and name != args.only:
            continue
        out = run_case(name, spec)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **out)
        e = out["expected"]
        print(f"{name}: expected {e.shape} range [{e.min():.3f}, {e.max():.3f}] -> {path}")


if __name__ == "__main__":
    main()
