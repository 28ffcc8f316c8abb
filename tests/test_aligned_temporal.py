"""Temporal NAFNet with deformable alignment (``aligned.AlignedTemporal``):
feature conv -> offset/mask conv on concat(centre, neighbour) -> DCNv2 per
neighbour -> 1x1 fusion + centre frame -> NAFNet trunk, against the same
wiring composed from the oracle's restatements
(oracle/nafnet_oracle.py:aligned_temporal_forward).

Inputs follow the temporal-alignment workload: T = 5 frames of one seeded
smooth base translated by integer shifts in [-4, 4] px, each with N(0, 20/255)
noise; 64 feature channels, 8 deformable groups, offsets of about N(0, 2 px).
Bar: max |out - fp32| <= 5e-3 and PSNR >= 50 dB, as for the model parity."""
import importlib
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
from parity_util import MAX_ABS, MIN_PSNR, compare, synth_mod  # noqa: E402

import nafnet_oracle as O  # noqa: E402


def oracle_case(pkg, tmp_path, cfg, t, h, w, seed):
    synth = synth_mod(pkg)
    apath, pa = synth.make_align_dir(str(tmp_path / "align"), seed, num_frames=t)
    tpath, pt = synth.make_model_dir(str(tmp_path / "trunk"), cfg, seed)
    clip = synth.temporal_window(t, h, w, seed).astype(np.float16).astype(np.float32)
    torch.set_num_threads(min(16, os.cpu_count() or 1))
    ref, oms = O.aligned_temporal_forward(O.as_torch(pa), O.as_torch(pt), torch.from_numpy(clip))
    return apath, tpath, clip, ref.numpy(), oms


def test_oracle_wiring_statistics(pkg, tmp_path):
    """The synthetic alignment weights give offsets of about N(0, 2 px) and
    masks spread around 0.5 on the synthetic window (CPU, oracle only)."""
    synth = synth_mod(pkg)
    _, _, clip, ref, oms = oracle_case(pkg, tmp_path, synth.CONFIG_TINY_W16, 5, 48, 64, seed=2)
    assert ref.shape == (1, 3, 48, 64) and np.isfinite(ref).all()
    n_off = 2 * synth.ALIGN_DG * 9
    assert len(oms) == 4 and all(om.shape == (1, 3 * synth.ALIGN_DG * 9, 48, 64) for om in oms)
    off = torch.cat([om[:, :n_off] for om in oms]).flatten()
    msk = torch.sigmoid(torch.cat([om[:, n_off:] for om in oms])).flatten()
    assert 1.2 <= float(off.std()) <= 3.5, float(off.std())
    assert 0.35 <= float(msk.mean()) <= 0.65 and float(msk.std()) >= 0.1


def test_oracle_wiring_matches_torchvision_composition(pkg, tmp_path):
    """The oracle's composition equals the same wiring built from torch's
    conv2d and torchvision's deform_conv2d (third-party DCNv2, mask = sigmoid
    of the raw masks, offsets [dy, dx] per (group, tap)) on the synthetic
    window (CPU). The offsets come from a conv of noisy features, so no sample
    lands exactly on the integer border positions where the two bilinear rules
    differ; measured agreement is ~2e-7."""
    tv = pytest.importorskip("torchvision")
    import torch.nn.functional as F

    synth = synth_mod(pkg)
    _, pa = synth.make_align_dir(str(tmp_path / "align"), 5, num_frames=5)
    _, pt = synth.make_model_dir(str(tmp_path / "trunk"), synth.CONFIG_TINY_W16, 5)
    clip = torch.from_numpy(synth.temporal_window(5, 32, 48, 5))
    pa_t, pt_t = O.as_torch(pa), O.as_torch(pt)
    torch.set_num_threads(min(16, os.cpu_count() or 1))
    ref, _ = O.aligned_temporal_forward(pa_t, pt_t, clip)

    conv = lambda k, x, pad: F.conv2d(x, pa_t[k + ".weight"], pa_t[k + ".bias"], padding=pad)  # noqa: E731
    t, c = 5, 2
    feats = [conv("align.feat", clip[:, i], 1) for i in range(t)]
    n_off = 2 * synth.ALIGN_DG * 9
    aligned = []
    for i in range(t):
        if i == c:
            aligned.append(feats[c])
            continue
        om = conv("align.offset", torch.cat([feats[c], feats[i]], 1), 1)
        aligned.append(tv.ops.deform_conv2d(feats[i], om[:, :n_off], pa_t["align.dcn.weight"], pa_t["align.dcn.bias"],
                                            padding=(1, 1), mask=torch.sigmoid(om[:, n_off:])))
    fused = conv("align.fuse", torch.cat(aligned, 1), 0) + clip[:, c]
    out = O.nafnet_forward(pt_t, fused)
    err = float((out - ref).abs().max())
    assert err <= 1e-4, err


@pytest.mark.gpu
@pytest.mark.parametrize("h,w", [(64, 96), (50, 70)], ids=["64x96", "50x70"])
def test_aligned_w32_matches_oracle(pkg, tmp_path, h, w):
    synth = synth_mod(pkg)
    aligned = importlib.import_module(pkg.__name__ + ".aligned")
    apath, tpath, clip, ref, _ = oracle_case(pkg, tmp_path, synth.CONFIG_W32, 5, h, w, seed=2)
    model = aligned.AlignedTemporal(apath, tpath)
    assert (model.num_frames, model.feat_channels, model.deform_groups) == (5, 64, 8)
    y = model(torch.from_numpy(clip).half().cuda())
    model.sync()
    err, psnr = compare(y.float().cpu().numpy(), ref)
    model.close()
    assert err <= MAX_ABS and psnr >= MIN_PSNR, (err, psnr)


@pytest.mark.gpu
def test_aligned_repeat_and_side_stream(pkg, tmp_path):
    """Two calls give identical outputs, on the current stream and on a side stream."""
    synth = synth_mod(pkg)
    aligned = importlib.import_module(pkg.__name__ + ".aligned")
    apath, _ = synth.make_align_dir(str(tmp_path / "align"), 3, num_frames=3)
    tpath, _ = synth.make_model_dir(str(tmp_path / "trunk"), synth.CONFIG_TINY_W16, 3)
    model = aligned.AlignedTemporal(apath, tpath)
    clip = torch.from_numpy(synth.temporal_window(3, 40, 56, 3)).half().cuda()
    a = model(clip)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    b = model(clip, stream=s)
    s.synchronize()
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    model.close()


def test_aligned_rejects_frames_beyond_the_layer_limit(pkg):
    """A window whose fusion input (T*F*H*W) exceeds 2^31 elements is rejected
    on the host before any kernel (2160x3840 at T = 5, F = 64). Host logic
    only: the instance skips layer construction and the clip is a meta tensor."""
    aligned = importlib.import_module(pkg.__name__ + ".aligned")
    m = aligned.AlignedTemporal.__new__(aligned.AlignedTemporal)
    m.num_frames, m.in_channels, m.feat_channels = 5, 3, 64
    clip = torch.empty(1, 5, 3, 2160, 3840, dtype=torch.float16, device="meta")
    with pytest.raises(ValueError, match="2\\^31"):
        m(clip)
    assert 5 * 64 * 1088 * 1920 <= aligned.MAX_LAYER_ELEMS  # 1080p windows stay within it


@pytest.mark.gpu
def test_aligned_rejects_bad_windows(pkg, tmp_path):
    synth = synth_mod(pkg)
    aligned = importlib.import_module(pkg.__name__ + ".aligned")
    apath, _ = synth.make_align_dir(str(tmp_path / "align"), 4, num_frames=3)
    tpath, _ = synth.make_model_dir(str(tmp_path / "trunk"), synth.CONFIG_TINY_W16, 4)
    model = aligned.AlignedTemporal(apath, tpath)
    with pytest.raises(ValueError):
        model(torch.zeros(1, 5, 3, 32, 32, dtype=torch.float16, device="cuda"))
    with pytest.raises(TypeError):
        model(torch.zeros(1, 3, 3, 32, 32, dtype=torch.float32, device="cuda"))
    model.close()
