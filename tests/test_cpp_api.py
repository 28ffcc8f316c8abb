"""The C++ API mirror (include/denoiser/: Tensor, WeightStore, Conv2dLayer,
DeformConv2dLayer, UpsampleLayer, NAFNet, NAFNetTemporal, kernels::launch_*)
compiles against the library like the reference's C++ callers, and behaves
like the reference headers: host-side checks on the CPU, the reference's
conv known answers and a NAFNet forward on the GPU."""
import os
import shutil
import subprocess

import numpy as np
import pytest

from parity_util import synth_mod

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "ml-video-denoiser_b200")
CUDA = "/usr/local/cuda"


def build_api_test(tmp_path):
    exe = os.path.join(str(tmp_path), "api_test")
    cmd = ["g++", "-std=c++20", "-O1", "-Wall", "-I", os.path.join(ROOT, "include"), "-I", f"{CUDA}/include",
           os.path.join(ROOT, "tests", "cpp", "api_test.cc"), "-L", PKG, "-ldenoiser_b200", "-L", f"{CUDA}/lib64",
           "-lcudart", f"-Wl,-rpath,{PKG}", f"-Wl,-rpath,{CUDA}/lib64", "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    return exe


def kat_manifest(pkg, d):
    synth = synth_mod(pkg)
    os.makedirs(d, exist_ok=True)
    params = {"conv1x1.weight": np.full((1, 1, 1, 1), 2.0, np.float16), "conv1x1.bias": np.ones(1, np.float16),
              "conv_multi.weight": np.array([1.0, -1.0], np.float16).reshape(2, 1, 1, 1)}
    return synth.write_manifest(d, params, {"type": "nafnet_residual", "base_channels": 32, "num_levels": 1,
                                           "in_channels": 1, "out_channels": 1, "enc_channels": [32]})


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ not available")
def test_cpp_api_compiles_and_host_checks_pass(pkg, tmp_path):
    pkg.lib()  # the library is built
    exe = build_api_test(tmp_path)
    man = kat_manifest(pkg, os.path.join(str(tmp_path), "kat"))
    r = subprocess.run([exe, "host", man], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.gpu
def test_cpp_api_on_gpu(pkg, tmp_path):
    import torch

    exe = build_api_test(tmp_path)
    man = kat_manifest(pkg, os.path.join(str(tmp_path), "kat"))
    synth = synth_mod(pkg)
    mdir = os.path.join(str(tmp_path), "model")
    os.makedirs(mdir, exist_ok=True)
    mpath, _ = synth.make_model_dir(mdir, synth.CONFIG_TINY_W16, 0)
    N, C, H, W = 1, 3, 70, 90
    x = synth.gradient_sinusoid_input(H, W, 3).astype(np.float16)
    assert x.shape == (N, C, H, W)
    m = pkg.Model(mpath)
    y = m(torch.from_numpy(x).cuda())
    m.sync()
    xb = os.path.join(str(tmp_path), "x.bin")
    yb = os.path.join(str(tmp_path), "y.bin")
    x.tofile(xb)
    y.cpu().numpy().astype(np.float16).tofile(yb)
    m.close()
    r = subprocess.run([exe, "gpu", man, mpath, xb, yb, str(N), str(C), str(H), str(W)], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
