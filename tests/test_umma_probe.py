"""tcgen05 descriptor conventions: one-tile GEMM against torch fp32."""
import pytest

torch = pytest.importorskip("torch")


@pytest.mark.gpu
@pytest.mark.parametrize("n,k", [(16, 16), (64, 32), (64, 64), (128, 128), (256, 64), (96, 256)])
def test_umma_probe_matches_fp32(pkg, n, k):
    g = torch.Generator(device="cpu").manual_seed(n * 1000 + k)
    a = torch.randn(128, k, generator=g).half().cuda()
    b = torch.randn(n, k, generator=g).half().cuda()
    d = pkg.umma_probe(a, b)
    ref = a.float() @ b.float().t()
    err = (d - ref).abs().max().item()
    assert err < 1e-2 * max(1.0, k / 64), err
