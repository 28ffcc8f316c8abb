"""dn_launch_global_avg_pool_noalloc (static device scratch, no allocation)
against dn_launch_global_avg_pool, both called through the C-ABI, and
against the numpy oracle.

Collected last on purpose: it must hold both in a fresh process, where its
first call does the per-device set-up, and after every other test."""
import ctypes
import os
import sys

import numpy as np
import pytest
import torch

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import kernels_oracle as ko  # noqa: E402

# the parity tolerance of the NCHW launcher tests against the oracle: 1 FP16 ulp
ULPS = 1

# 2049 planes x 128 splits (any H*W above 127 * 16384) need 262272 split sums,
# above the 262144 the static scratch holds.
TOO_BIG = (1, 2049, 1088, 1920)


def ulp_close(a, b, ulps=ULPS):
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    tol = ulps * np.maximum(np.abs(b), 2.0 ** -14) * 2.0 ** -10
    return bool(np.all(np.abs(a - b) <= tol + 1e-12))


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(1, 32, 544, 960), (2, 64, 130, 250), (3, 5, 7, 9)])
def test_noalloc_pool_matches_allocating_pool(pkg, shape):
    lib = pkg.lib()
    N, C, H, W = shape
    xh = np.random.default_rng(21).uniform(0, 1, size=shape).astype(np.float16)
    x = torch.from_numpy(xh).cuda()
    want = torch.empty((N, C), dtype=torch.float16, device="cuda")
    pkg.check(lib.dn_launch_global_avg_pool(x.data_ptr(), want.data_ptr(), N, C, H, W, _stream()))
    torch.cuda.synchronize()
    ref = want.cpu().numpy()
    # the same plan, kernels and summation order: bit-identical results
    for _ in range(2):  # two calls in a row reuse the same static scratch
        got = torch.full((N, C), float("nan"), dtype=torch.float16, device="cuda")
        pkg.check(lib.dn_launch_global_avg_pool_noalloc(x.data_ptr(), got.data_ptr(), N, C, H, W, _stream()))
        torch.cuda.synchronize()
        g = got.cpu().numpy()
        assert np.array_equal(g.view(np.int16), ref.view(np.int16))
        # and within the launcher tolerance of the oracle's sequential sum
        assert ulp_close(g, ko.global_avg_pool(xh))


@pytest.mark.gpu
def test_noalloc_pool_rejects_sizes_beyond_its_scratch(pkg):
    lib = pkg.lib()
    # a buffer of the claimed size, so that even a broken size rule reads in bounds
    N, C, H, W = TOO_BIG
    t = torch.zeros(N * C * H * W, dtype=torch.float16, device="cuda")
    out = torch.zeros(N * C, dtype=torch.float16, device="cuda")
    rc = lib.dn_launch_global_avg_pool_noalloc(t.data_ptr(), out.data_ptr(), N, C, H, W, _stream())
    if rc == pkg.DN_OK:
        torch.cuda.synchronize()
    assert rc == pkg.DN_ERR_UNSUPPORTED
    assert b"static scratch" in lib.dn_last_error()
    del t


@pytest.mark.skipif(torch.cuda.is_available(), reason="host-only check; fake pointers stay off GPU machines")
def test_noalloc_pool_size_rule_is_host_only(pkg):
    """The rejection happens before any CUDA call, so it runs without a GPU:
    the pointers are never dereferenced."""
    lib = pkg.lib()
    N, C, H, W = TOO_BIG
    rc = lib.dn_launch_global_avg_pool_noalloc(ctypes.c_void_p(256), ctypes.c_void_p(512), N, C, H, W, None)
    assert rc == pkg.DN_ERR_UNSUPPORTED
    assert b"static scratch" in lib.dn_last_error()
