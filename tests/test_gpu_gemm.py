"""The projection variant's tcgen05 product (sparc_proj_gemm) against a float32 torch reference
of the same bfloat16 operands: float32 output to 1e-5 relative l2 (accumulation order only),
bfloat16 output to 1e-2 (its rounding), fused skip and rank-2 terms included."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30))


@pytest.mark.parametrize("rows,n,k", [(128, 128, 64), (300, 200, 520), (1000, 64, 64), (16384, 512, 512),
                                      (7, 9, 8), (4096, 1024, 128)])
def test_gemm_matches_torch(rows, n, k):
    from sparc_b200 import gemm

    g = torch.Generator(device="cuda").manual_seed(rows + n + k)
    a = torch.randn(rows, k, generator=g, device="cuda").bfloat16()
    b = torch.randn(n, k, generator=g, device="cuda").bfloat16()
    ref = a.float() @ b.float().t()
    out32 = gemm.proj_gemm(a, b, torch.float32)
    out16 = gemm.proj_gemm(a, b, torch.bfloat16)
    torch.cuda.synchronize()
    assert gemm.gemm_status("cuda") == 0
    assert _rel(out32, ref) < 1e-5
    assert _rel(out16.float(), ref) < 1e-2


def test_gemm_fused_terms():
    from sparc_b200 import gemm

    rows, n, k = 777, 320, 192
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(rows, k, generator=g, device="cuda").bfloat16()
    b = torch.randn(n, k, generator=g, device="cuda").bfloat16()
    x = torch.randn(rows, n, generator=g, device="cuda").bfloat16()
    skip = torch.randn(n, generator=g, device="cuda")
    dp = torch.randn(rows, 2, generator=g, device="cuda")
    c0 = torch.randn(n, generator=g, device="cuda")
    c1 = torch.randn(n, generator=g, device="cuda")
    ref = a.float() @ b.float().t() + skip * x.float() + dp[:, :1] * c0 + dp[:, 1:] * c1
    out = gemm.proj_gemm(a, b, torch.float32, x=x, skip=skip, dp=dp, c0=c0, c1=c1)
    assert _rel(out, ref) < 1e-5
    out = gemm.proj_gemm(a, b, torch.float32, x=x, skip=skip)
    assert _rel(out, a.float() @ b.float().t() + skip * x.float()) < 1e-5
    assert gemm.gemm_status("cuda") == 0


@pytest.mark.parametrize("rows,n,k", [(300, 200, 520), (16384, 512, 512)])
def test_gemm_f32_split(rows, n, k):
    """float32 operands through the three-term bf16 split: ~1e-5 of a float64 product."""
    from sparc_b200 import gemm

    g = torch.Generator(device="cuda").manual_seed(rows + k)
    a = torch.randn(rows, k, generator=g, device="cuda")
    b = torch.randn(n, k, generator=g, device="cuda")
    dp = torch.randn(rows, 2, generator=g, device="cuda")
    c0 = torch.randn(n, generator=g, device="cuda")
    c1 = torch.randn(n, generator=g, device="cuda")
    ref = a.double() @ b.double().t() + dp[:, :1].double() * c0.double() + dp[:, 1:].double() * c1.double()
    out = gemm.proj_gemm_f32(a, b, dp=dp, c0=c0, c1=c1)
    assert _rel(out, ref) < 5e-5
    assert gemm.gemm_status("cuda") == 0
