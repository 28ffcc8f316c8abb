"""dn_launch_global_avg_pool_noalloc (static device scratch, no allocation)
against dn_launch_global_avg_pool, both called through the C-ABI.

Collected last on purpose: it must hold both in a fresh process, where its
first call does the per-device set-up, and after every other test."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

# the parity tolerance of the NCHW launcher tests: 1 FP16 ulp
ULPS = 1


def ulp_close(a, b, ulps=ULPS):
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    tol = ulps * np.maximum(np.abs(b), 2.0 ** -14) * 2.0 ** -10
    return bool(np.all(np.abs(a - b) <= tol + 1e-12))


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("shape", [(1, 32, 544, 960), (2, 64, 130, 250), (3, 5, 7, 9)])
def test_noalloc_pool_matches_allocating_pool(pkg, shape):
    lib = pkg.lib()
    N, C, H, W = shape
    x = torch.from_numpy(np.random.default_rng(21).uniform(0, 1, size=shape).astype(np.float16)).cuda()
    want = torch.empty((N, C), dtype=torch.float16, device="cuda")
    pkg.check(lib.dn_launch_global_avg_pool(x.data_ptr(), want.data_ptr(), N, C, H, W, _stream()))
    torch.cuda.synchronize()
    ref = want.cpu().numpy()
    for _ in range(2):  # two calls in a row reuse the same static scratch
        got = torch.full((N, C), float("nan"), dtype=torch.float16, device="cuda")
        pkg.check(lib.dn_launch_global_avg_pool_noalloc(x.data_ptr(), got.data_ptr(), N, C, H, W, _stream()))
        torch.cuda.synchronize()
        assert ulp_close(got.cpu().numpy(), ref)


def test_noalloc_pool_rejects_sizes_beyond_its_scratch(pkg):
    lib = pkg.lib()
    t = torch.zeros(16, dtype=torch.float16, device="cuda")
    # 2049 planes x 128 splits (1088x1920) needs 262272 split sums > 262144
    rc = lib.dn_launch_global_avg_pool_noalloc(t.data_ptr(), t.data_ptr(), 1, 2049, 1088, 1920, _stream())
    assert rc == pkg.DN_ERR_UNSUPPORTED
    assert b"static scratch" in lib.dn_last_error()
