"""DeformConv2dLayer (fused DCNv2 kernel) against the golden vector produced
by torchvision.ops.deform_conv2d and against the CPU oracle
(oracle/nafnet_oracle.py:deform_conv2d, a restatement of
src/kernels/deform_im2col.cuh:34-142 + the GEMM of
src/layers/deform_conv2d.cu:134-182).

Bar: max |out - fp32| <= 5e-3 and PSNR >= 50 dB, as for the model parity."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
from parity_util import MAX_ABS, MIN_PSNR, compare, load_golden, synth_mod  # noqa: E402

import nafnet_oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu


def make_layer(pkg, tmp_path, weight, bias, **kw):
    import importlib

    synth = synth_mod(pkg)
    params = {"dcn.weight": weight.astype(np.float16)}
    if bias is not None:
        params["dcn.bias"] = bias.astype(np.float16)
    path = synth.write_manifest(str(tmp_path), params, {"type": "dcn"})
    layers = importlib.import_module(pkg.__name__ + ".layers")
    store = pkg.Weights(path)
    return layers.DeformConv2d(store, "dcn.weight", "dcn.bias" if bias is not None else None, **kw), store


def run(layer, x, off, msk):
    out = layer(torch.from_numpy(x).half().cuda(), torch.from_numpy(off).half().cuda(),
                torch.from_numpy(msk).half().cuda())
    layer.sync()
    return out.float().cpu().numpy()


def test_dcn_matches_reference_golden(pkg, tmp_path):
    g = load_golden("dcn_c16_dg4_20x24")
    meta = g["meta"]
    layer, _ = make_layer(pkg, tmp_path, g["weight"], g["bias"], pad=meta["pad"], stride=meta["stride"],
                          dilation=meta["dilation"], deform_groups=meta["dg"])
    assert (layer.out_channels, layer.in_channels, layer.deform_groups) == (16, 16, 4)
    y = run(layer, g["x"], g["offsets"], g["masks"])
    err, psnr = compare(y, g["expected"])
    assert err <= MAX_ABS and psnr >= MIN_PSNR, (err, psnr)


CASES = [
    # cin, cout, dg, n, h, w, pad, stride, dilation
    (64, 64, 8, 2, 33, 47, 1, 1, 1),
    (64, 40, 8, 1, 30, 36, 1, 2, 1),
    (32, 32, 4, 1, 25, 31, 2, 1, 2),
    (32, 48, 32, 1, 17, 19, 1, 1, 1),
    (16, 256, 2, 1, 20, 24, 1, 1, 1),
]


@pytest.mark.parametrize("cin,cout,dg,n,h,w,pad,stride,dil", CASES)
def test_dcn_matches_oracle(pkg, tmp_path, cin, cout, dg, n, h, w, pad, stride, dil):
    rng = np.random.default_rng(cin * 7 + cout + dg)
    q = lambda a: a.astype(np.float16).astype(np.float32)  # noqa: E731
    ho = (h + 2 * pad - dil * 2 - 1) // stride + 1
    wo = (w + 2 * pad - dil * 2 - 1) // stride + 1
    x = q(rng.uniform(-1, 1, (n, cin, h, w)))
    off = rng.normal(0, 2.0, (n, 2 * dg * 9, ho, wo))
    off = q(np.where(np.abs(off - np.round(off)) < 0.02, off + 0.05, off))
    msk = q(rng.normal(0, 1.5, (n, dg * 9, ho, wo)))
    bound = 1.0 / np.sqrt(cin * 9)
    wt = q(rng.uniform(-bound, bound, (cout, cin, 3, 3)))
    bs = q(rng.uniform(-bound, bound, (cout,)))
    layer, _ = make_layer(pkg, tmp_path, wt, bs, pad=pad, stride=stride, dilation=dil, deform_groups=dg)
    y = run(layer, x, off, msk)
    torch.set_num_threads(min(16, os.cpu_count() or 1))
    ref = O.deform_conv2d(torch.from_numpy(x), torch.from_numpy(off), torch.from_numpy(msk), torch.from_numpy(wt),
                          torch.from_numpy(bs), pad=pad, stride=stride, dilation=dil, deform_groups=dg).numpy()
    assert y.shape == ref.shape
    err, psnr = compare(y, ref)
    assert err <= MAX_ABS and psnr >= MIN_PSNR, (err, psnr)


def test_dcn_repeat_is_deterministic(pkg, tmp_path):
    g = load_golden("dcn_c16_dg4_20x24")
    layer, _ = make_layer(pkg, tmp_path, g["weight"], g["bias"], deform_groups=4)
    a = run(layer, g["x"], g["offsets"], g["masks"])
    b = run(layer, g["x"], g["offsets"], g["masks"])
    assert np.array_equal(a, b)


def test_dcn_errors(pkg, tmp_path):
    g = load_golden("dcn_c16_dg4_20x24")
    with pytest.raises(pkg.NotFoundError):
        make_layer(pkg, tmp_path, g["weight"], g["bias"])[0].__class__(
            pkg.Weights(os.path.join(str(tmp_path), "manifest.json")), "missing.weight", None)
    with pytest.raises(pkg.InvalidArgumentError):
        make_layer(pkg, tmp_path, g["weight"], g["bias"], deform_groups=5)
    layer, _ = make_layer(pkg, tmp_path, g["weight"], g["bias"], deform_groups=4)
    with pytest.raises(TypeError):
        layer(torch.zeros(1, 16, 20, 24, device="cuda"), torch.zeros(1, 72, 20, 24, device="cuda").half(),
              torch.zeros(1, 36, 20, 24, device="cuda").half())
