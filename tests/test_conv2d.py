"""Conv2dLayer (implicit-GEMM kernel) against the reference's own conv
known-answer tests (tests/test_conv2d.cc:34-268: 1x1 weight 2.0 with and
without bias 1.0 on inputs 1..9, two output channels +1/-1, padding grows a
1x1 output, accessors) and against torch.nn.functional.conv2d in FP32 on the
CPU for 3x3, 2x2 stride 2, depthwise, grouped, dilated and > 256-channel
layers.

Bar: max |out - fp32| <= 5e-3 and PSNR >= 50 dB, as for the model parity."""
import importlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.nn.functional as F  # noqa: E402
from parity_util import MAX_ABS, MIN_PSNR, compare, synth_mod  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L(pkg):
    return importlib.import_module(pkg.__name__ + ".layers")


def store_of(pkg, tmp_path, params):
    synth = synth_mod(pkg)
    path = synth.write_manifest(str(tmp_path), {k: v.astype(np.float16) for k, v in params.items()},
                               {"type": "nafnet_residual", "base_channels": 32, "num_levels": 1, "in_channels": 1})
    return pkg.Weights(path)


def fp16_dev(a):
    return torch.from_numpy(np.asarray(a, dtype=np.float16)).cuda()


def run(layer, x):
    y = layer(fp16_dev(x))
    layer.sync()
    return y.float().cpu().numpy()


@pytest.fixture
def kat_store(pkg, tmp_path):
    # the reference fixture: conv1x1 = 2.0 (+ bias 1.0), conv_multi = [1, -1]
    return store_of(pkg, tmp_path, {"conv1x1.weight": np.full((1, 1, 1, 1), 2.0), "conv1x1.bias": np.ones(1),
                                    "conv_multi.weight": np.array([1.0, -1.0]).reshape(2, 1, 1, 1)})


def test_kat_1x1_no_bias(L, kat_store):
    conv = L.Conv2d(kat_store, "conv1x1.weight", None, pad=0)
    y = run(conv, np.arange(1, 10, dtype=np.float32).reshape(1, 1, 3, 3))
    assert y.shape == (1, 1, 3, 3)
    assert np.allclose(y.ravel(), 2.0 * np.arange(1, 10), atol=1e-2)


def test_kat_1x1_with_bias(L, kat_store):
    conv = L.Conv2d(kat_store, "conv1x1.weight", "conv1x1.bias", pad=0)
    y = run(conv, np.arange(1, 10, dtype=np.float32).reshape(1, 1, 3, 3))
    assert np.allclose(y.ravel(), 2.0 * np.arange(1, 10) + 1.0, atol=1e-2)


def test_kat_multi_channel(L, kat_store):
    conv = L.Conv2d(kat_store, "conv_multi.weight", None, pad=0)
    y = run(conv, np.arange(1, 5, dtype=np.float32).reshape(1, 1, 2, 2))
    assert y.shape == (1, 2, 2, 2)
    assert np.allclose(y[0, 0].ravel(), [1, 2, 3, 4], atol=1e-2)
    assert np.allclose(y[0, 1].ravel(), [-1, -2, -3, -4], atol=1e-2)


def test_kat_padding_grows_1x1_output(L, kat_store):
    conv = L.Conv2d(kat_store, "conv1x1.weight", None, pad=1)
    y = run(conv, np.ones((1, 1, 3, 3), dtype=np.float32))
    assert y.shape == (1, 1, 5, 5)


def test_kat_accessors_and_errors(pkg, L, kat_store):
    conv = L.Conv2d(kat_store, "conv1x1.weight", None, pad=0)
    assert (conv.out_channels, conv.in_channels, conv.kernel_h, conv.kernel_w) == (1, 1, 1, 1)
    multi = L.Conv2d(kat_store, "conv_multi.weight", None, pad=0)
    assert (multi.out_channels, multi.in_channels) == (2, 1)
    with pytest.raises(TypeError):
        conv(torch.ones(1, 1, 3, 3, device="cuda"))
    with pytest.raises(pkg.NotFoundError):
        L.Conv2d(kat_store, "missing.weight")
    # repeated calls on one size reuse the layer's buffers
    x = fp16_dev(np.ones((1, 1, 3, 3)))
    conv(x)
    conv(x)
    conv.sync()


CASES = [
    # cout, cin_g, k, pad, stride, dil, groups, n, h, w
    (32, 3, 3, 1, 1, 1, 1, 1, 37, 53),      # intro-like 3x3
    (3, 32, 3, 1, 1, 1, 1, 2, 24, 20),      # ending-like 3x3
    (64, 32, 2, 0, 2, 1, 1, 1, 30, 44),     # 2x2 stride-2 downsample
    (64, 1, 3, 1, 1, 1, 64, 1, 33, 47),     # depthwise
    (48, 8, 3, 1, 1, 1, 4, 1, 20, 28),      # grouped
    (32, 16, 3, 2, 1, 2, 1, 1, 25, 31),     # dilated
    (300, 64, 1, 0, 1, 1, 1, 1, 17, 23),    # > 256 outputs: two slabs
    (16, 24, 5, 2, 2, 1, 1, 1, 19, 27),     # 5x5 stride 2, Cin not a power of two
]


@pytest.mark.parametrize("cout,cin_g,k,pad,stride,dil,groups,n,h,w", CASES)
def test_conv_matches_torch(pkg, L, tmp_path, cout, cin_g, k, pad, stride, dil, groups, n, h, w):
    rng = np.random.default_rng(cout * 31 + cin_g * 7 + k)
    q = lambda a: a.astype(np.float16).astype(np.float32)  # noqa: E731
    bound = 1.0 / np.sqrt(cin_g * k * k)
    wt = q(rng.uniform(-bound, bound, (cout, cin_g, k, k)))
    bs = q(rng.uniform(-bound, bound, (cout,)))
    x = q(rng.uniform(-1, 1, (n, cin_g * groups, h, w)))
    store = store_of(pkg, tmp_path, {"c.weight": wt, "c.bias": bs})
    conv = L.Conv2d(store, "c.weight", "c.bias", pad=pad, stride=stride, dilation=dil, groups=groups)
    assert conv.groups == groups
    y = run(conv, x)
    ref = F.conv2d(torch.from_numpy(x), torch.from_numpy(wt), torch.from_numpy(bs), stride=stride, padding=pad,
                   dilation=dil, groups=groups).numpy()
    assert y.shape == ref.shape
    err, psnr = compare(y, ref)
    assert err <= MAX_ABS and psnr >= MIN_PSNR, (err, psnr)
