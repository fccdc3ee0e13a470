"""The projection variant's tcgen05 product (sparc_proj_gemm) against a float32 torch reference
of the same bfloat16 operands: float32 output to 1e-5 relative l2 (accumulation order only),
bfloat16 output to 1e-2 (its rounding), fused skip and rank-2 terms included."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30))


@pytest.mark.parametrize("rows,n,k", [(128, 128, 64), (300, 200, 520), (1000, 64, 64), (16384, 512, 512),
                                      (7, 9, 8), (4096, 1024, 128),
                                      # several output tiles per CTA (the tensor-memory reuse)
                                      (65536, 1024, 256), (40000, 777, 136)])
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


@pytest.mark.parametrize("rows,n,k", [(777, 320, 192), (30001, 1000, 64)])
def test_gemm_fused_terms(rows, n, k):
    from sparc_b200 import gemm

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


@pytest.mark.parametrize("a_mn,b_mn", [(True, True), (True, False), (False, True)])
@pytest.mark.parametrize("rows,n,k", [(128, 256, 64), (200, 136, 1000), (2048, 2048, 16384), (8, 8, 7)])
def test_gemm_token_major_operands(rows, n, k, a_mn, b_mn):
    """Operands stored transposed (a [k, rows], b [k, n]: the weight gradients x^T du and dy^T h
    over the tokens) against the float64 product of the same bf16 values; k not a multiple of
    64 (zero-filled tail) and output tiles cut at the edges. The float32 accumulation's error
    grows like sqrt(k): 1e-5 relative l2 up to k = 1024, 1e-5 sqrt(k / 1024) beyond."""
    from sparc_b200 import gemm

    g = torch.Generator(device="cuda").manual_seed(rows * 3 + n + k)
    at = torch.randn(k, rows, generator=g, device="cuda").bfloat16()  # [k, rows]
    bt = torch.randn(k, n, generator=g, device="cuda").bfloat16()     # [k, n]
    ref = at.double().t() @ bt.double()
    a = at if a_mn else at.t().contiguous()
    b = bt if b_mn else bt.t().contiguous()
    if (not a_mn or not b_mn) and k % 8:
        pytest.skip("a K-major operand needs k a multiple of 8")
    out = gemm.proj_gemm(a, b, torch.float32, a_mn=a_mn, b_mn=b_mn)
    torch.cuda.synchronize()
    assert gemm.gemm_status("cuda") == 0
    assert _rel(out, ref) < 1e-5 * max(1.0, (k / 1024) ** 0.5)


def test_gemm_token_major_f32_split():
    """float32 weight gradients through the split along the tokens: ~1e-5 of float64."""
    from sparc_b200 import gemm

    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(3000, 64, generator=g, device="cuda")
    du = torch.randn(3000, 128, generator=g, device="cuda")
    ref = x.double().t() @ du.double()
    out = gemm.proj_gemm_f32(x, du, a_mn=True, b_mn=True)
    assert _rel(out, ref) < 5e-5 and out.shape == (64, 128)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows,w", [(16384, 2048), (1000, 10), (3, 700), (777, 6144), (50, 64), (1001, 512),
                                    (9, 16384)])
def test_colsum_and_rowdot(rows, w, dtype):
    """The layer's skinny products: x^T dp with the bias row and sum dy x per column (fixed
    order), and p = x c + bias per row, against float64 torch; widths that take the 16-byte
    vector kernels with one to eight warps per row and one to four column chunks per thread,
    widths that do not (10; 700 in bfloat16), and rows not a multiple of a CTA's rows."""
    from sparc_b200 import gemm

    g = torch.Generator(device="cuda").manual_seed(rows + w)
    x = torch.randn(rows, w, generator=g, device="cuda").to(dtype)
    dy = torch.randn(rows, w, generator=g, device="cuda").to(dtype)
    dp = torch.randn(rows, 2, generator=g, device="cuda")
    c = torch.randn(w + 1, 2, generator=g, device="cuda")
    d_ctl, d_skip = gemm.proj_colsum(x, dp, dy)
    xd, dyd, dpd = x.double(), dy.double(), dp.double()
    assert _rel(d_ctl[:w], xd.t() @ dpd) < 1e-5 and _rel(d_ctl[w], dpd.sum(0)) < 1e-5
    assert _rel(d_skip, (dyd * xd).sum(0)) < 1e-5
    d_ctl2, none = gemm.proj_colsum(x, dp)
    assert none is None and torch.equal(d_ctl2, d_ctl)  # bitwise reproducible
    p = gemm.proj_rowdot(x, c)
    assert _rel(p, xd @ c[:w].double() + c[w].double()) < 1e-5
