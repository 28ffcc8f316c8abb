"""Tiled inference with ramp blending and temporal flip averaging
(training/infer.py:174-281 of the reference): the oracle restatement against
golden vectors written by the reference's own functions (CPU), and the
engine (ml-video-denoiser_b200/infer.py over include/denoiser_b200_infer.h)
against the same vectors (GPU). Bar for the engine: max |out - fp32| <= 5e-3
and PSNR >= 50 dB, as for the model parity."""
import importlib
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
from parity_util import MAX_ABS, MIN_PSNR, compare, golden_model_dir, load_golden, synth_mod  # noqa: E402

import infer_oracle as IO  # noqa: E402
import nafnet_oracle as O  # noqa: E402

TILE = ["tile_spatial_w16_70x90_t32"]
FLIP = ["flip_temporal_py_w8_t3_seq5", "flip_temporal_py_w8_t3_seq4_t16"]


def _params(pkg, tmp_path, meta):
    m = dict(meta)
    m["kind"] = {"tile_spatial": "spatial", "flip_temporal": "temporal_py"}[meta["kind"]]
    return golden_model_dir(pkg, tmp_path, m)


def test_ramp_matches_reference_rule():
    r = IO.make_ramp(6, 9, 4)[0, 0]
    lin = torch.linspace(0, 1, 4)
    ry = torch.tensor([lin[0], lin[1], lin[3], lin[2], lin[1], lin[0]])  # the reversed ramp wins where they meet
    rx = torch.tensor([lin[0], lin[1], lin[2], lin[3], 1.0, lin[3], lin[2], lin[1], lin[0]])
    assert torch.equal(r, ry[:, None] * rx[None, :])
    with pytest.raises(RuntimeError):
        IO.make_ramp(3, 9, 4)


@pytest.mark.parametrize("name", TILE)
def test_oracle_tiles_match_reference(pkg, tmp_path, name):
    g = load_golden(name)
    _, params = _params(pkg, tmp_path, g["meta"])
    p = O.as_torch(params)
    y = IO.tile_inference(lambda t: O.nafnet_forward(p, t), torch.from_numpy(g["x"]), g["meta"]["tile"])
    assert float((y - torch.from_numpy(g["expected"])).abs().max()) <= 2e-5


@pytest.mark.parametrize("name", FLIP)
def test_oracle_flip_matches_reference(pkg, tmp_path, name):
    g = load_golden(name)
    _, params = _params(pkg, tmp_path, g["meta"])
    p = O.as_torch(params)
    frames = [torch.from_numpy(f) for f in g["x"]]
    ys = IO.denoise_temporal_sequence(lambda c: O.nafnet_temporal_forward(p, c), frames, g["meta"]["frames"],
                                      True, g["meta"]["tile"])
    assert float((torch.stack(ys) - torch.from_numpy(g["expected"])).abs().max()) <= 2e-5


@pytest.mark.gpu
@pytest.mark.parametrize("name", TILE)
def test_engine_tiles_match_reference(pkg, tmp_path, name):
    infer = importlib.import_module(pkg.__name__ + ".infer")
    g = load_golden(name)
    path, _ = _params(pkg, tmp_path, g["meta"])
    m = pkg.Model(path)
    y = infer.tile_inference(m, torch.from_numpy(g["x"]).half().cuda(), g["meta"]["tile"])
    m.sync()
    err, psnr = compare(y.float().cpu().numpy(), g["expected"])
    m.close()
    assert err <= MAX_ABS and psnr >= MIN_PSNR, (err, psnr)


@pytest.mark.gpu
@pytest.mark.parametrize("name", FLIP)
def test_engine_flip_matches_reference(pkg, tmp_path, name):
    infer = importlib.import_module(pkg.__name__ + ".infer")
    g = load_golden(name)
    path, _ = _params(pkg, tmp_path, g["meta"])
    m = pkg.Model(path)
    frames = [torch.from_numpy(f).half().cuda() for f in g["x"]]
    ys = infer.denoise_temporal_sequence(m, frames, g["meta"]["frames"], True, g["meta"]["tile"])
    m.sync()
    err, psnr = compare(torch.stack(ys).float().cpu().numpy(), g["expected"])
    m.close()
    assert err <= MAX_ABS and psnr >= MIN_PSNR, (err, psnr)


@pytest.mark.gpu
def test_engine_tiles_at_1080p_match_oracle(pkg, tmp_path):
    """NAFNet-w32 on a 1080p frame in 512-pixel tiles (overlap 64, stride
    448: 3 x 5 tiles, ragged at the right and bottom edges) against the
    oracle's tiled inference of the same frame; the frame's outermost row
    and column are 0, as the reference's ramps make them."""
    synth = synth_mod(pkg)
    infer = importlib.import_module(pkg.__name__ + ".infer")
    path, params = synth.make_model_dir(str(tmp_path), synth.CONFIG_W32, 1)
    m = pkg.Model(path)
    x = synth.w32_frame(1080, 1920, seed=3).astype(np.float16).astype(np.float32)
    y = infer.tile_inference(m, torch.from_numpy(x).half().cuda(), 512)
    m.sync()
    got = y.float().cpu().numpy()
    m.close()
    assert np.all(got[..., 0, :] == 0) and np.all(got[..., :, 0] == 0)
    assert np.all(got[..., -1, :] == 0) and np.all(got[..., :, -1] == 0)
    torch.set_num_threads(min(16, os.cpu_count() or 1))
    p = O.as_torch(params)
    ref = IO.tile_inference(lambda t: O.nafnet_forward(p, t), torch.from_numpy(x), 512).numpy()
    err, psnr = compare(got, ref)
    assert err <= MAX_ABS and psnr >= MIN_PSNR, (err, psnr)


@pytest.mark.gpu
def test_engine_rejects_tiles_narrower_than_the_overlap(pkg, tmp_path):
    synth = synth_mod(pkg)
    infer = importlib.import_module(pkg.__name__ + ".infer")
    cfg = synth.NAFConfig(base_channels=8, enc_blocks=(1, 1), middle_blocks=1, dec_blocks=(1, 1))
    path, _ = synth.make_model_dir(str(tmp_path), cfg, 0)
    m = pkg.Model(path)
    # tile 64: overlap 8, stride 56; the last column of tiles is 6 wide (the
    # 2-level model pads it to 8 and runs it), narrower than the overlap
    x = torch.zeros(1, 3, 64, 62, dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError, match="narrower"):
        infer.tile_inference(m, x, 64)
    m.close()
