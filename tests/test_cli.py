"""The `denoiser` command-line tool (ml-video-denoiser_b200/cli/denoiser.cc):
the reference CLI's flags and outputs (cli/main.cc:43-58, 133-136, 254-256,
329-331), frame sharding over --gpus N, and the reference's own cli/main.cc
compiled unchanged against this repository's include/ (the C++ boundary).

GPU runs read and write EXR (HALF channels), so the files hold the engine's
FP16 outputs exactly and the comparisons are bit for bit."""
import importlib
import os
import shutil
import subprocess

import numpy as np
import pytest

from parity_util import synth_mod

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "ml-video-denoiser_b200", "denoiser")
REF_CLI = os.path.join(ROOT, "oracle", "_ref", "ref_cli_on_engine")
REFERENCE = os.environ.get("DENOISER_REFERENCE", "/root/reference")


def run(args, timeout=300):
    return subprocess.run([str(a) for a in args], capture_output=True, text=True, timeout=timeout)


@pytest.fixture(scope="module")
def cli(pkg):
    if not os.path.exists(CLI):
        r = subprocess.run(["make", "-C", os.path.dirname(CLI), "denoiser"], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr[-2000:]
    return CLI


def test_cli_usage_and_argument_errors(cli):
    r = run([cli, "--help"])
    assert r.returncode == 0 and "--model" in r.stderr and "--gpus" in r.stderr
    r = run([cli])
    assert r.returncode == 1 and "Usage:" in r.stderr
    r = run([cli, "--model", "m.json", "--input", "x.png", "--bogus"])
    assert r.returncode == 1 and "unknown flag: --bogus" in r.stderr
    r = run([cli, "--input", "x.png"])
    assert r.returncode == 1 and "--model is required" in r.stderr
    r = run([cli, "--model", "m.json", "--input", "x.png", "--frames"])
    assert r.returncode == 1 and "missing value for --frames" in r.stderr


@pytest.mark.skipif(not os.path.isdir(os.path.join(REFERENCE, "cli")) or shutil.which("g++") is None,
                    reason="reference sources not present")
def test_reference_cli_source_builds_against_include(pkg, tmp_path):
    """The reference's cli/main.cc compiles and links, unchanged, against
    include/ (Tensor, WeightStore, NAFNet, NAFNetTemporal, io::*) and the
    engine library: a C++ caller of the reference switches by recompiling."""
    pkg.lib()
    exe = str(tmp_path / "ref_cli")
    lib_dir = os.path.join(ROOT, "ml-video-denoiser_b200")
    r = run(["g++", "-std=c++20", "-O1", "-I", os.path.join(ROOT, "include"), "-I", "/usr/local/cuda/include",
             os.path.join(REFERENCE, "cli", "main.cc"), "-o", exe, "-L", lib_dir, "-ldenoiser_b200",
             "-L", "/usr/local/cuda/lib64", "-lcudart", f"-Wl,-rpath,{lib_dir}"], timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    r = run([exe, "--help"])
    assert r.returncode == 0 and "--prefetch" in r.stderr


def write_frames(pkg, d, frames):
    io = importlib.import_module(pkg.__name__ + ".image_io")
    os.makedirs(d, exist_ok=True)
    names = []
    for i, f in enumerate(frames):
        name = f"frame_{i:04d}.exr"
        io.save(os.path.join(d, name), f.astype(np.float16))
        names.append(name)
    return names


@pytest.mark.gpu
@pytest.mark.parametrize("gpus", [1, 2])
def test_cli_spatial_directory_matches_model(pkg, cli, tmp_path, gpus):
    import torch

    if gpus > torch.cuda.device_count():
        pytest.skip(f"needs {gpus} GPUs")
    synth = synth_mod(pkg)
    io = importlib.import_module(pkg.__name__ + ".image_io")
    path, _ = synth.make_model_dir(str(tmp_path / "m"), synth.CONFIG_TINY_W16, 0)
    frames = [synth.gradient_sinusoid_input(40, 56, seed=i)[0] for i in range(5)]
    names = write_frames(pkg, str(tmp_path / "in"), frames)
    r = run([cli, "--model", path, "--input", tmp_path / "in", "--gpus", gpus])
    assert r.returncode == 0, r.stdout + r.stderr
    assert f"Processing {len(names)} images" in r.stdout
    out_dir = tmp_path / "in_denoised"  # the reference's default (<input>_denoised)
    m = pkg.Model(path)
    for name in names:
        x = io.load(str(tmp_path / "in" / name))
        want = m(torch.from_numpy(x).cuda())
        m.sync()
        got = io.load(str(out_dir / name))
        assert np.array_equal(got.view(np.int16), want.cpu().numpy().view(np.int16)), name
    m.close()


@pytest.mark.gpu
@pytest.mark.parametrize("gpus", [1, 2])
def test_cli_temporal_directory_matches_sharded_model(pkg, cli, tmp_path, gpus):
    """Temporal mode (edge replication, cli/main.cc:163-174) through the frame
    cache, split over --gpus segments with halos: equal to a single-rank run
    of the engine over the same frames."""
    import torch

    if gpus > torch.cuda.device_count():
        pytest.skip(f"needs {gpus} GPUs")
    synth = synth_mod(pkg)
    io = importlib.import_module(pkg.__name__ + ".image_io")
    sharding = importlib.import_module(pkg.__name__ + ".sharding")
    cfg = synth.NAFConfig(base_channels=8, enc_blocks=(1, 1), middle_blocks=1, dec_blocks=(1, 1), dw_expand=1,
                          ffn_expand=2)
    path, _ = synth.make_model_dir(str(tmp_path / "m"), cfg, 3, "legacy", 3, True)
    seq = synth.temporal_window(7, 32, 48, seed=3)[0]
    names = write_frames(pkg, str(tmp_path / "in"), list(seq))
    out_dir = tmp_path / "out"
    r = run([cli, "--model", path, "--input", tmp_path / "in", "--output", out_dir, "--mode", "temporal",
             "--gpus", gpus])
    assert r.returncode == 0, r.stdout + r.stderr
    m = pkg.Model(path)
    held = [torch.from_numpy(io.load(str(tmp_path / "in" / n))[0]).cuda() for n in names]
    want = sharding.denoise_segment(m, lambda i: held[i], len(names), 1, 0, num_frames=3)
    m.sync()
    for (i, y), name in zip(want, names):
        got = io.load(str(out_dir / name))[0]
        assert np.array_equal(got.view(np.int16), y.cpu().numpy().view(np.int16)), name
    m.close()


@pytest.mark.gpu
def test_cli_single_image_default_output(pkg, cli, tmp_path):
    import torch

    synth = synth_mod(pkg)
    io = importlib.import_module(pkg.__name__ + ".image_io")
    path, _ = synth.make_model_dir(str(tmp_path / "m"), synth.CONFIG_TINY_W16, 1)
    img = tmp_path / "shot.exr"
    io.save(str(img), synth.gradient_sinusoid_input(37, 53, seed=9))
    r = run([cli, "--model", path, "--input", img, "--prefetch"])
    assert r.returncode == 0, r.stdout + r.stderr
    out = tmp_path / "shot_denoised.exr"
    assert f"Saved: {out}" in r.stdout
    m = pkg.Model(path)
    want = m(torch.from_numpy(io.load(str(img))).cuda())
    m.sync()
    assert np.array_equal(io.load(str(out)).view(np.int16), want.cpu().numpy().view(np.int16))
    m.close()


@pytest.mark.gpu
@pytest.mark.skipif(not os.path.exists(REF_CLI), reason="oracle/_ref/ref_cli_on_engine not built")
def test_reference_cli_binary_runs_on_the_engine(pkg, cli, tmp_path):
    """The reference's own main.cc (built by oracle/Makefile against include/)
    denoises a directory through the engine with the same results as this
    repository's CLI."""
    synth = synth_mod(pkg)
    io = importlib.import_module(pkg.__name__ + ".image_io")
    path, _ = synth.make_model_dir(str(tmp_path / "m"), synth.CONFIG_TINY_W16, 2)
    names = write_frames(pkg, str(tmp_path / "in"), [synth.gradient_sinusoid_input(32, 40, seed=i)[0]
                                                     for i in range(3)])
    r1 = run([REF_CLI, "--model", path, "--input", tmp_path / "in", "--output", tmp_path / "a"])
    r2 = run([cli, "--model", path, "--input", tmp_path / "in", "--output", tmp_path / "b"])
    assert r1.returncode == 0 and r2.returncode == 0, r1.stderr + r2.stderr
    for n in names:
        assert np.array_equal(io.load(str(tmp_path / "a" / n)), io.load(str(tmp_path / "b" / n)))
