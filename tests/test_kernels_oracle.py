"""Pins the NCHW launcher oracle (oracle/kernels_oracle.py) to torch's CPU
operators, the ones the reference's PyTorch model uses for the same steps
(training/models.py: F.pad reflect in _pad_to_multiple, nn.PixelShuffle,
LayerNorm2d, AdaptiveAvgPool2d, SimpleGate, grid_sample border)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import kernels_oracle as ko


def rng_half(shape, seed, lo=-1.0, hi=1.0):
    r = np.random.default_rng(seed)
    return r.uniform(lo, hi, size=shape).astype(np.float16)


def ulp_close(a, b, ulps=1):
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    tol = ulps * np.maximum(np.abs(b), 2.0 ** -14) * 2.0 ** -10
    return bool(np.all(np.abs(a - b) <= tol + 1e-12))


@pytest.mark.parametrize("shape,pad", [((1, 3, 13, 17), (3, 2)), ((2, 4, 8, 8), (7, 7)), ((1, 1, 5, 1), (4, 0))])
def test_reflect_pad_matches_torch(shape, pad):
    x = rng_half(shape, 1)
    ph, pw = pad
    want = F.pad(torch.from_numpy(x).float(), (0, pw, 0, ph), mode="reflect").half().numpy()
    got = ko.reflect_pad(x, shape[2] + ph, shape[3] + pw)
    assert np.array_equal(got, want)


def test_pixel_shuffle_matches_torch():
    x = rng_half((2, 12, 5, 7), 2)
    want = F.pixel_shuffle(torch.from_numpy(x).float(), 2).half().numpy()
    assert np.array_equal(ko.pixel_shuffle2x(x), want)


def test_layer_norm_matches_torch():
    x = rng_half((2, 24, 6, 9), 3, -3, 3)
    w = np.random.default_rng(4).uniform(0.5, 1.5, 24).astype(np.float32)
    b = np.random.default_rng(5).uniform(-0.2, 0.2, 24).astype(np.float32)
    t = torch.from_numpy(x).float().permute(0, 2, 3, 1)
    want = F.layer_norm(t, (24,), torch.from_numpy(w), torch.from_numpy(b), eps=1e-6)
    want = want.permute(0, 3, 1, 2).half().numpy()
    assert ulp_close(ko.layer_norm_affine(x, w, b), want, ulps=2)


def test_global_avg_pool_matches_torch():
    x = rng_half((2, 5, 33, 47), 6, 0, 1)
    want = torch.from_numpy(x).float().mean(dim=(2, 3)).half().numpy()
    assert ulp_close(ko.global_avg_pool(x), want, ulps=1)


def test_simple_gate_matches_chunk_and_flat_at_n1():
    x = rng_half((2, 8, 4, 5), 7)
    a, b = torch.from_numpy(x).float().chunk(2, dim=1)
    want = (a * b).half().numpy()
    assert np.array_equal(ko.simple_gate(x), want)
    x1 = x[:1]
    assert np.array_equal(ko.simple_gate_flat(x1, 1, 4, 4, 5), ko.simple_gate(x1))


def test_warp_matches_grid_sample_border():
    N, C, H, W = 1, 3, 9, 11
    f = rng_half((N, C, H, W), 8)
    off = rng_half((N, 2, H, W), 9, -3, 3)
    ft = torch.from_numpy(f).float()
    o = torch.from_numpy(off).float()
    hh, ww = torch.meshgrid(torch.arange(H).float(), torch.arange(W).float(), indexing="ij")
    gx = 2 * (ww + o[:, 0]) / (W - 1) - 1
    gy = 2 * (hh + o[:, 1]) / (H - 1) - 1
    want = F.grid_sample(ft, torch.stack([gx, gy], dim=-1), mode="bilinear", padding_mode="border",
                         align_corners=True)
    got = ko.warp_bilinear(f, off).astype(np.float32)
    assert np.max(np.abs(got - want.numpy())) < 2e-3


def test_elementwise_and_copies():
    a = rng_half((2, 3, 4, 5), 10)
    b = rng_half((2, 3, 4, 5), 11)
    assert np.array_equal(ko.add(a, b), (torch.from_numpy(a).float() + torch.from_numpy(b).float()).half().numpy())
    sc = ko.subtract_clamp(a, b)
    assert sc.min() >= 0 and sc.max() <= 1
    assert np.array_equal(ko.concat_channels(a, b), torch.cat([torch.from_numpy(a), torch.from_numpy(b)], 1).numpy())
    assert np.array_equal(ko.crop(a, 2, 3), a[:, :, :2, :3])
    clip = rng_half((2, 5, 3, 4, 4), 12)
    assert np.array_equal(ko.extract_frame(clip, 3), clip[:, 3])
    assert np.array_equal(ko.select_prefix_channels(a, 2), a[:, :2])
    s = rng_half((2, 3), 13)
    want = (torch.from_numpy(a).float() * torch.from_numpy(s).float()[:, :, None, None]).half().numpy()
    assert np.array_equal(ko.mul_channelwise(a, s), want)


def test_upsample_matches_torch_away_from_the_low_border():
    # The reference kernel extrapolates on the first output row/column
    # (unclamped weight); elsewhere it is PyTorch's align_corners=False bilinear.
    x = rng_half((1, 3, 7, 9), 14)
    want = F.interpolate(torch.from_numpy(x).float(), scale_factor=2, mode="bilinear",
                         align_corners=False).half().numpy()
    got = ko.upsample_bilinear(x, 2)
    assert got.shape == want.shape
    assert ulp_close(got[:, :, 1:, 1:], want[:, :, 1:, 1:], ulps=1)
    # first output row: source row -0.25 -> weights 1.25 / -0.25 on input rows 0 / 1
    # (columns from 1 on, where the horizontal weights are PyTorch's)
    def hrow(r):
        return F.interpolate(torch.from_numpy(x[:, :, r:r + 1, :]).float(), scale_factor=(1, 2),
                             mode="bilinear", align_corners=False).numpy()[:, :, 0, :]
    expect = 1.25 * hrow(0) - 0.25 * hrow(1)
    assert np.allclose(got[:, :, 0, 1:].astype(np.float32), expect[:, :, 1:], atol=2e-3)
