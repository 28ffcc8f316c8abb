"""Engine vs the reference's own C++ FP16 engine, run on the same GPU.

The reference engine (src/models/nafnet.cu, nafnet_temporal.cu,
src/layers/conv2d.cu, deform_conv2d.cu with cuDNN and cuBLAS) is built
unchanged by oracle/Makefile into oracle/_ref/ref_engine, a test-only
harness; these tests run it as a subprocess on files of seeded FP16 inputs
and compare its output with the engine's on the same inputs and weights.

Bar: max |engine - reference FP16 engine| <= 5e-3 per pixel and PSNR >= 50 dB,
the reference's own parity threshold (tests/test_unet_forward.cc:207). It
holds for DeformConv2dLayer too, although the reference's GEMM there is
cublasHgemm with FP16 accumulation (src/layers/deform_conv2d.cu:156-168)
and the engine accumulates in FP32.
"""
import importlib
import json
import os
import subprocess

import numpy as np
import pytest

torch = pytest.importorskip("torch")
from parity_util import MAX_ABS, MIN_PSNR, compare, synth_mod  # noqa: E402

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_ENGINE = os.path.join(ROOT, "oracle", "_ref", "ref_engine")

need_ref = pytest.mark.skipif(not os.path.exists(REF_ENGINE),
                              reason="oracle/_ref/ref_engine not built (make -C oracle)")


def ref_run(args, timeout=900):
    """Run the reference-engine harness; returns its stdout."""
    r = subprocess.run([REF_ENGINE] + [str(a) for a in args], capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, f"reference engine failed ({r.returncode}): {r.stderr.strip()}"
    return r.stdout


def f16_file(tmp_path, name, a):
    p = os.path.join(str(tmp_path), name)
    np.ascontiguousarray(a.astype(np.float16)).tofile(p)
    return p


def read_f16(path, shape):
    return np.fromfile(path, dtype=np.float16).reshape(shape).astype(np.float32)


def engine_forward(pkg, path, x):
    m = pkg.Model(path)
    y = m(torch.from_numpy(x).half().cuda())
    m.sync()
    out = y.float().cpu().numpy()
    m.close()
    return out


def ref_nafnet(tmp_path, path, x):
    xin = f16_file(tmp_path, "x.f16", x)
    out = os.path.join(str(tmp_path), "y_ref.f16")
    n, c, h, w = x.shape
    ref_run(["nafnet", path, xin, n, c, h, w, out])
    return read_f16(out, (n, 3, h, w))


def _spatial_case(pkg, tmp_path, cfg, seed, x):
    synth = synth_mod(pkg)
    path, _ = synth.make_model_dir(str(tmp_path), cfg, seed)
    y_ref = ref_nafnet(tmp_path, path, x)
    y = engine_forward(pkg, path, x)
    return compare(y, y_ref)


@need_ref
def test_tiny_w16_256_vs_reference_engine(pkg, tmp_path):
    """Tiny NAFNet w16 (4 levels of 1 block), 1x3x256x256, seed 0."""
    synth = synth_mod(pkg)
    x = synth.gradient_sinusoid_input(256, 256, seed=0).astype(np.float16).astype(np.float32)
    err, psnr = _spatial_case(pkg, tmp_path, synth.CONFIG_TINY_W16, 0, x)
    print(f"vs reference engine: max abs {err:.3e}, PSNR {psnr:.2f} dB")
    assert err <= MAX_ABS and psnr >= MIN_PSNR, (err, psnr)


@need_ref
def test_w32_ragged_vs_reference_engine(pkg, tmp_path):
    """NAFNet-w32, a size that needs reflect padding and a crop (100x150)."""
    synth = synth_mod(pkg)
    x = synth.w32_frame(100, 150, seed=5).astype(np.float16).astype(np.float32)
    err, psnr = _spatial_case(pkg, tmp_path, synth.CONFIG_W32, 1, x)
    print(f"vs reference engine: max abs {err:.3e}, PSNR {psnr:.2f} dB")
    assert err <= MAX_ABS and psnr >= MIN_PSNR, (err, psnr)


@need_ref
def test_w32_literal_expansion_1080p_vs_reference_engine(pkg, tmp_path):
    """NAFNet-w32 with dw_expand=2 / ffn_expand=2 (the repo-literal reading of
    "expansion 2", 64.68 M params) on one 1080p frame."""
    synth = synth_mod(pkg)
    x = synth.w32_frame(1080, 1920, seed=3).astype(np.float16).astype(np.float32)
    err, psnr = _spatial_case(pkg, tmp_path, synth.CONFIG_W32_LITERAL, 3, x)
    print(f"vs reference engine: max abs {err:.3e}, PSNR {psnr:.2f} dB")
    assert err <= MAX_ABS and psnr >= MIN_PSNR, (err, psnr)


@need_ref
def test_w32_1080p_vs_reference_engine(pkg, tmp_path):
    """NAFNet-w32 on one 1080p Poisson-Gaussian frame, seed-1 weights (the
    benchmark workload)."""
    synth = synth_mod(pkg)
    x = synth.w32_frame(1080, 1920, seed=1).astype(np.float16).astype(np.float32)
    err, psnr = _spatial_case(pkg, tmp_path, synth.CONFIG_W32, 1, x)
    print(f"vs reference engine: max abs {err:.3e}, PSNR {psnr:.2f} dB")
    assert err <= MAX_ABS and psnr >= MIN_PSNR, (err, psnr)


@need_ref
@pytest.mark.parametrize("frames,warp,hw", [(3, True, (64, 96)), (5, False, (50, 70)), (5, True, (136, 240))])
def test_legacy_temporal_vs_reference_engine(pkg, tmp_path, frames, warp, hw):
    """The reference C++ NAFNetTemporal design (temporal_mix.N on
    concat(ref, mean(warped neighbours)), 1x1 offset heads with the pixel
    warp) on a seeded w16 export."""
    synth = synth_mod(pkg)
    cfg = synth.NAFConfig(base_channels=16, enc_blocks=(1, 1, 2), middle_blocks=2, dec_blocks=(1, 1, 1),
                          dw_expand=1, ffn_expand=2)
    path, _ = synth.make_model_dir(str(tmp_path), cfg, 3, "legacy", frames, warp)
    h, w = hw
    clip = synth.temporal_window(frames, h, w, seed=4).astype(np.float16).astype(np.float32)
    xin = f16_file(tmp_path, "clip.f16", clip)
    out = os.path.join(str(tmp_path), "y_ref.f16")
    ref_run(["temporal", path, xin, 1, frames, 3, h, w, out])
    y_ref = read_f16(out, (1, 3, h, w))
    y = engine_forward(pkg, path, clip)
    err, psnr = compare(y, y_ref)
    print(f"vs reference engine: max abs {err:.3e}, PSNR {psnr:.2f} dB")
    assert err <= MAX_ABS and psnr >= MIN_PSNR, (err, psnr)


def _dcn_case(pkg, tmp_path, cin, cout, dg, h, w, seed):
    synth = synth_mod(pkg)
    layers = importlib.import_module(pkg.__name__ + ".layers")
    rng = np.random.default_rng(seed)
    bound = 1.0 / np.sqrt(cin * 9)
    params = {"dcn.weight": rng.uniform(-bound, bound, (cout, cin, 3, 3)).astype(np.float32),
              "dcn.bias": rng.uniform(-bound, bound, (cout,)).astype(np.float32)}
    path = synth.write_manifest(str(tmp_path), params, {"type": "dcn"})
    x = rng.uniform(-1, 1, (1, cin, h, w)).astype(np.float16)
    off = rng.normal(0.0, 2.0, (1, 2 * dg * 9, h, w)).astype(np.float16)
    msk = rng.normal(0.0, 1.0, (1, dg * 9, h, w)).astype(np.float16)
    files = [f16_file(tmp_path, n, a) for n, a in (("x.f16", x), ("off.f16", off), ("msk.f16", msk))]
    out = os.path.join(str(tmp_path), "y_ref.f16")
    ref_run(["dcn", path, "dcn.weight", "dcn.bias", files[0], 1, cin, h, w, files[1], files[2], 1, 1, 1, dg, out])
    y_ref = read_f16(out, (1, cout, h, w))
    store = pkg.Weights(path)
    layer = layers.DeformConv2d(store, "dcn.weight", "dcn.bias", pad=1, stride=1, dilation=1, deform_groups=dg)
    y = layer(torch.from_numpy(x).cuda(), torch.from_numpy(off).cuda(), torch.from_numpy(msk).cuda())
    layer.sync()
    return compare(y.float().cpu().numpy(), y_ref)


@need_ref
@pytest.mark.parametrize("h,w", [(45, 67), (1080, 1920)])
def test_dcn_vs_reference_engine(pkg, tmp_path, h, w):
    """DeformConv2dLayer 3x3, 64 -> 64 channels, 8 deformable groups, offsets
    N(0, 2 px) and raw masks N(0, 1): the alignment layer of the temporal
    model with deformable alignment, up to its 1080p size."""
    err, psnr = _dcn_case(pkg, tmp_path, 64, 64, 8, h, w, seed=h)
    print(f"vs reference engine: max abs {err:.3e}, PSNR {psnr:.2f} dB")
    assert err <= MAX_ABS and psnr >= MIN_PSNR, (err, psnr)


CONV_CASES = [
    # cout, cin/groups, k, pad, stride, groups, h, w: the convolution shapes of NAFNet
    (32, 3, 3, 1, 1, 1, 67, 91),     # intro
    (3, 32, 3, 1, 1, 1, 40, 56),     # ending
    (64, 1, 3, 1, 1, 64, 45, 61),    # depthwise (cuDNN grouped conv, groups = C)
    (64, 32, 2, 0, 2, 1, 44, 60),    # 2x2 stride-2 downsample
    (512, 256, 1, 0, 1, 1, 34, 60),  # 1x1 conv at the middle level
]


@need_ref
@pytest.mark.parametrize("cout,cin_g,k,pad,stride,groups,h,w", CONV_CASES)
def test_conv2d_vs_reference_engine(pkg, tmp_path, cout, cin_g, k, pad, stride, groups, h, w):
    """Conv2dLayer (the reference's cuDNN implicit-precomp GEMM + bias)."""
    synth = synth_mod(pkg)
    layers = importlib.import_module(pkg.__name__ + ".layers")
    rng = np.random.default_rng(cout + 7 * k + groups)
    bound = 1.0 / np.sqrt(cin_g * k * k)
    params = {"c.weight": rng.uniform(-bound, bound, (cout, cin_g, k, k)).astype(np.float32),
              "c.bias": rng.uniform(-bound, bound, (cout,)).astype(np.float32)}
    path = synth.write_manifest(str(tmp_path), params, {"type": "conv"})
    x = rng.uniform(-1, 1, (1, cin_g * groups, h, w)).astype(np.float16)
    xin = f16_file(tmp_path, "x.f16", x)
    out = os.path.join(str(tmp_path), "y_ref.f16")
    ref_run(["conv", path, "c.weight", "c.bias", xin, 1, cin_g * groups, h, w, pad, stride, 1, groups, out])
    ho, wo = (h + 2 * pad - k) // stride + 1, (w + 2 * pad - k) // stride + 1
    y_ref = read_f16(out, (1, cout, ho, wo))
    store = pkg.Weights(path)
    conv = layers.Conv2d(store, "c.weight", "c.bias", pad=pad, stride=stride, dilation=1, groups=groups)
    y = conv(torch.from_numpy(x).cuda())
    conv.sync()
    err, psnr = compare(y.float().cpu().numpy(), y_ref)
    print(f"vs reference engine: max abs {err:.3e}, PSNR {psnr:.2f} dB")
    assert err <= MAX_ABS and psnr >= MIN_PSNR, (err, psnr)


@need_ref
def test_reference_engine_timing_line(pkg, tmp_path):
    """The harness's timing mode (used by bench.py) prints one JSON object."""
    synth = synth_mod(pkg)
    path, _ = synth.make_model_dir(str(tmp_path), synth.CONFIG_TINY_W16, 0)
    x = synth.gradient_sinusoid_input(64, 96, seed=0).astype(np.float16)
    xin = f16_file(tmp_path, "x.f16", x)
    out = os.path.join(str(tmp_path), "y.f16")
    line = ref_run(["nafnet", path, xin, 1, 3, 64, 96, out, 2]).strip().splitlines()[-1]
    d = json.loads(line)
    assert d["reps"] == 2 and d["ms"] > 0
