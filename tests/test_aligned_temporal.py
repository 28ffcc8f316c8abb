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
@pytest.mark.parametrize("h,w", [(64, 96), (50, 70), (256, 448)], ids=["64x96", "50x70", "256x448"])
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


@pytest.mark.gpu
def test_alignment_stage_1080p_matches_oracle(pkg, tmp_path):
    """The alignment stage (trunk input) of a 5-frame 1080p window, 64
    features, 8 deformable groups, against the oracle's composition. The
    engine aligns the whole frame; the oracle runs on row bands with a
    32-row margin (the features, the offset conv and every deformable sample
    of the compared rows lie inside the band: offsets are about N(0, 2 px)),
    at the top and bottom borders and in the middle."""
    synth = synth_mod(pkg)
    aligned = importlib.import_module(pkg.__name__ + ".aligned")
    h, w, t = 1080, 1920, 5
    apath, pa = synth.make_align_dir(str(tmp_path / "align"), 2, num_frames=t)
    tpath, _ = synth.make_model_dir(str(tmp_path / "trunk"), synth.CONFIG_TINY_W16, 2)
    clip = synth.temporal_window(t, h, w, seed=2).astype(np.float16).astype(np.float32)
    model = aligned.AlignedTemporal(apath, tpath)
    xc = torch.from_numpy(clip).half().cuda()
    for i in range(t):
        model.encode_frame(xc[:, i], i)
    fused = model.align_window(list(range(t)), h, w)
    model.sync()
    got = fused.float().cpu().numpy()
    model.close()
    torch.set_num_threads(min(16, os.cpu_count() or 1))
    pa_t = O.as_torch(pa)
    for lo, hi, c0, c1 in ((0, 96, 0, 64), (500, 628, 532, 596), (984, 1080, 1016, 1080)):
        ref, _ = O.aligned_fusion(pa_t, torch.from_numpy(clip[:, :, :, lo:hi]))
        ref = ref.numpy()[:, :, c0 - lo:c1 - lo]
        err, psnr = compare(got[:, :, c0:c1], ref)
        assert err <= MAX_ABS and psnr >= MIN_PSNR, ((lo, hi), err, psnr)


@pytest.mark.gpu
def test_frame_cache_matches_window_forward(pkg, tmp_path):
    """A sequence through the frame cache (each frame encoded once, slot
    f % T, edge replication by repeated slots) equals one forward per
    assembled window, bit for bit."""
    synth = synth_mod(pkg)
    aligned = importlib.import_module(pkg.__name__ + ".aligned")
    sharding = importlib.import_module(pkg.__name__ + ".sharding")
    t, n, h, w = 5, 7, 40, 56
    apath, _ = synth.make_align_dir(str(tmp_path / "align"), 6, num_frames=t)
    tpath, _ = synth.make_model_dir(str(tmp_path / "trunk"), synth.CONFIG_TINY_W16, 6)
    model = aligned.AlignedTemporal(apath, tpath)
    seq = torch.from_numpy(synth.temporal_window(n, h, w, 6)[0]).half().cuda()
    cached = sharding.denoise_segment(model, lambda i: seq[i], n, 1, 0, num_frames=t)
    direct = sharding.denoise_segment(model, lambda i: seq[i], n, 1, 0, num_frames=t, cache=False)
    model.sync()
    assert [i for i, _ in cached] == list(range(n))
    for (_, a), (_, b) in zip(cached, direct):
        assert torch.equal(a, b)
    model.close()


@pytest.mark.gpu
def test_aligned_rejects_frames_beyond_the_layer_limit(pkg, tmp_path):
    """A frame whose offset-conv output (3*dg*9 channels) would exceed 2^31
    elements is rejected on the host before any copy or kernel (4320x7680;
    2160x3840 is within the limit). The frame buffer has the full size."""
    synth = synth_mod(pkg)
    aligned = importlib.import_module(pkg.__name__ + ".aligned")
    apath, _ = synth.make_align_dir(str(tmp_path / "align"), 4, num_frames=3)
    tpath, _ = synth.make_model_dir(str(tmp_path / "trunk"), synth.CONFIG_TINY_W16, 4)
    model = aligned.AlignedTemporal(apath, tpath)
    big = torch.zeros(1, 3, 4320, 7680, dtype=torch.float16, device="cuda")
    with pytest.raises(pkg.DenoiserError, match="2\\^31"):
        model.encode_frame(big, 0)
    assert 216 * 2160 * 3840 < 2 ** 31
    model.close()
