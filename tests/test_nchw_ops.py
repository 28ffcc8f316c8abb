"""Parity of the NCHW launchers (include/denoiser_b200_ops.h) against the
numpy restatement of the reference kernels (oracle/kernels_oracle.py).

Copies must be bit-exact; element-wise arithmetic within 1 FP16 ulp (FP32 math
and one rounding on both sides, FMA contraction aside); reductions
(LayerNorm, average pool) within 2 ulps, since they add in another order.
Every op runs on the 16-byte vector path (aligned sizes) and on the scalar
path (odd sizes, or a pointer 2 bytes off alignment)."""
import numpy as np
import pytest
import torch

from oracle import kernels_oracle as ko

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K(pkg):
    import importlib

    return importlib.import_module(pkg.__name__ + ".kernels")


def rng_half(shape, seed, lo=-1.0, hi=1.0):
    return np.random.default_rng(seed).uniform(lo, hi, size=shape).astype(np.float16)


def dev(x, misalign=False):
    """Device copy of x; with misalign the data starts 2 bytes past a 16-byte boundary."""
    t = torch.from_numpy(np.ascontiguousarray(x))
    if not misalign:
        return t.cuda()
    buf = torch.empty(t.numel() + 8, dtype=t.dtype, device="cuda")
    v = buf[1:1 + t.numel()].view(t.shape)
    v.copy_(t.cuda())
    return v


def empty(shape, dtype=torch.float16, misalign=False):
    n = int(np.prod(shape))
    if not misalign:
        return torch.empty(shape, dtype=dtype, device="cuda")
    return torch.empty(n + 8, dtype=dtype, device="cuda")[1:1 + n].view(shape)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def ulp_close(a, b, ulps=1):
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    tol = ulps * np.maximum(np.abs(b), 2.0 ** -14) * 2.0 ** -10
    bad = np.abs(a - b) > tol + 1e-12
    return not bad.any(), int(bad.sum())


SHAPES = [((1, 32, 64, 96), False), ((2, 3, 13, 17), False), ((1, 8, 16, 24), True)]


@pytest.mark.parametrize("shape,mis", SHAPES)
def test_elementwise(K, shape, mis):
    a = rng_half(shape, 1)
    b = rng_half(shape, 2)
    n = a.size
    out = empty(shape, misalign=mis)
    K.launch_add(dev(a, mis), dev(b), out, n)
    ok, nbad = ulp_close(host(out), ko.add(a, b))
    assert ok, nbad
    K.launch_mul_scalar(dev(a, mis), 0.37, out, n)
    ok, nbad = ulp_close(host(out), ko.mul_scalar(a, 0.37))
    assert ok, nbad
    K.launch_subtract_clamp(dev(a * 2, mis), dev(b), out, n)
    assert np.array_equal(host(out), ko.subtract_clamp(a * 2, b))


@pytest.mark.parametrize("shape,mis", SHAPES)
def test_channel_ops(K, shape, mis):
    N, C, H, W = shape
    x = rng_half(shape, 3)
    r = rng_half(shape, 4)
    s16 = rng_half((N, C), 5)
    out = empty(shape, misalign=mis)
    K.launch_mul_channelwise(dev(x, mis), dev(s16), out, N, C, H, W)
    ok, nbad = ulp_close(host(out), ko.mul_channelwise(x, s16))
    assert ok, nbad
    for fp32 in (True, False):
        sc = np.random.default_rng(6).uniform(-1, 1, C).astype(np.float32 if fp32 else np.float16)
        K.launch_scaled_add(dev(x, mis), dev(r), dev(sc), fp32, out, N, C, H, W)
        ok, nbad = ulp_close(host(out), ko.scaled_add(x, r, sc))
        assert ok, nbad


@pytest.mark.parametrize("shape,mis", SHAPES)
def test_simple_gate(K, shape, mis):
    N, C, H, W = shape
    x = rng_half((N, 2 * C, H, W), 7)
    out = empty(shape, misalign=mis)
    K.launch_simple_gate(dev(x, mis), out, N, C, H, W)
    got = host(out)
    assert np.array_equal(got, ko.simple_gate(x))
    if N == 1:
        assert np.array_equal(got, ko.simple_gate_flat(x, N, C, H, W))


@pytest.mark.parametrize("shape,mis", SHAPES + [((1, 512, 17, 30), False), ((1, 1500, 5, 7), False)])
@pytest.mark.parametrize("fp32", [True, False])
def test_layer_norm(K, shape, mis, fp32):
    N, C, H, W = shape
    x = rng_half(shape, 8, -2, 3)
    dt = np.float32 if fp32 else np.float16
    w = np.random.default_rng(9).uniform(0.5, 1.5, C).astype(dt)
    b = np.random.default_rng(10).uniform(-0.3, 0.3, C).astype(dt)
    out = empty(shape, misalign=mis)
    K.launch_layer_norm_affine(dev(x, mis), dev(w), dev(b), fp32, out, N, C, H, W)
    ok, nbad = ulp_close(host(out), ko.layer_norm_affine(x, w, b), ulps=2)
    assert ok, nbad


@pytest.mark.parametrize("shape,mis", SHAPES + [((1, 32, 1088, 1920), False), ((3, 7, 1, 1), False)])
def test_global_avg_pool(K, shape, mis):
    N, C, H, W = shape
    x = rng_half(shape, 11, 0, 1)
    out = empty((N, C))
    K.launch_global_avg_pool(dev(x, mis), out, N, C, H, W)
    ok, nbad = ulp_close(host(out), ko.global_avg_pool(x), ulps=1)
    assert ok, nbad


def test_global_avg_pool_deterministic(K):
    x = dev(rng_half((1, 16, 300, 500), 12, 0, 1))
    o1, o2 = empty((1, 16)), empty((1, 16))
    K.launch_global_avg_pool(x, o1, 1, 16, 300, 500)
    K.launch_global_avg_pool(x, o2, 1, 16, 300, 500)
    assert torch.equal(o1, o2)


@pytest.mark.parametrize("shape,mis", SHAPES)
def test_pixel_shuffle(K, shape, mis):
    N, C, H, W = shape
    C4 = C * 4 if C % 4 else C
    x = rng_half((N, C4, H, W), 13)
    out = empty((N, C4 // 4, 2 * H, 2 * W), misalign=mis)
    K.launch_pixel_shuffle2x(dev(x), out, N, C4, H, W)
    assert np.array_equal(host(out), ko.pixel_shuffle2x(x))


@pytest.mark.parametrize("shape", [(1, 16, 40, 56), (2, 3, 13, 17)])
def test_warp_bilinear(K, shape):
    N, C, H, W = shape
    f = rng_half(shape, 14)
    off = rng_half((N, 2, H, W), 15, -4, 4)
    out = empty(shape)
    K.launch_warp_bilinear(dev(f), dev(off), out, N, C, H, W)
    got = host(out).astype(np.float32)
    want = ko.warp_bilinear(f, off).astype(np.float32)
    assert np.max(np.abs(got - want)) <= 2.0 ** -10 * 2


@pytest.mark.parametrize("shape,mis", SHAPES)
def test_copies(K, shape, mis):
    N, C, H, W = shape
    x = rng_half(shape, 16)
    ph, pw = min(H - 1, 8), min(W - 1, 8)
    out = empty((N, C, H + ph, W + pw), misalign=mis)
    K.launch_reflect_pad(dev(x, mis), out, N, C, H, W, H + ph, W + pw)
    padded = host(out)
    assert np.array_equal(padded, ko.reflect_pad(x, H + ph, W + pw))
    back = empty(shape, misalign=mis)
    K.launch_crop(dev(padded), back, N, C, H + ph, W + pw, H, W)
    assert np.array_equal(host(back), x)
    y = rng_half((N, 5, H, W), 17)
    cat = empty((N, C + 5, H, W), misalign=mis)
    K.launch_concat_channels(dev(x, mis), dev(y), cat, N, C, 5, H, W)
    assert np.array_equal(host(cat), ko.concat_channels(x, y))
    pre = empty((N, 2, H, W), misalign=mis)
    K.launch_select_prefix_channels(dev(x), pre, N, C, 2, H, W)
    assert np.array_equal(host(pre), ko.select_prefix_channels(x, 2))
    clip = rng_half((N, 5, C, H, W), 18)
    fr = empty(shape, misalign=mis)
    K.launch_extract_frame(dev(clip), fr, N, 5, C, H, W, 4)
    assert np.array_equal(host(fr), ko.extract_frame(clip, 4))


def test_reflect_pad_full_frame(K):
    x = rng_half((1, 3, 1080, 1920), 19)
    out = empty((1, 3, 1088, 1920))
    K.launch_reflect_pad(dev(x), out, 1, 3, 1080, 1920, 1088, 1920)
    assert np.array_equal(host(out), ko.reflect_pad(x, 1088, 1920))


def test_zero_sizes_are_noops(K, pkg):
    t = empty((4,))
    K.launch_add(t, t, t, 0)
    K.launch_global_avg_pool(t, t, 0, 3, 4, 4)
    K.launch_reflect_pad(t, t, 0, 3, 4, 4, 6, 6)
    K.launch_layer_norm_affine(t, t, t, True, t, 1, 4, 0, 5)
    torch.cuda.synchronize()


def test_invalid_arguments_raise(K, pkg):
    t = empty((64,))
    with pytest.raises(pkg.InvalidArgumentError):
        K.launch_reflect_pad(t, t, 1, 1, 4, 4, 8, 4)  # pad wider than the image
    with pytest.raises(pkg.InvalidArgumentError):
        K.launch_crop(t, t, 1, 1, 4, 4, 5, 4)
    with pytest.raises(pkg.InvalidArgumentError):
        K.launch_extract_frame(t, t, 1, 2, 1, 4, 4, 2)
    with pytest.raises(pkg.InvalidArgumentError):
        K.launch_pixel_shuffle2x(t, t, 1, 6, 2, 2)
    with pytest.raises(pkg.InvalidArgumentError):
        K.launch_add(t, t, t, -1)
    with pytest.raises(pkg.InvalidArgumentError):
        K.launch_global_avg_pool(t, t, 1, 2, 0, 4)
    with pytest.raises(pkg.InvalidArgumentError):
        K.launch_simple_gate(None, t, 1, 1, 4, 4)


@pytest.mark.parametrize("shape,scale", [((1, 8, 17, 23), 2), ((2, 3, 5, 7), 3), ((1, 32, 135, 240), 2)])
def test_upsample_bilinear(K, shape, scale):
    N, C, H, W = shape
    x = rng_half(shape, 20)
    out = empty((N, C, H * scale, W * scale))
    K.upsample_bilinear(dev(x), out, N, C, H, W, scale)
    ok, nbad = ulp_close(host(out), ko.upsample_bilinear(x, scale), ulps=1)
    assert ok, nbad


def test_upsample_rejects_bad_scale(K, pkg):
    t = empty((16,))
    with pytest.raises(pkg.InvalidArgumentError):
        K.upsample_bilinear(t, t, 1, 1, 2, 2, 0)
