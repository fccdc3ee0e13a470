"""The generic complex scans (sparc_b200.complex_scan, complex_scan_with_last) on the GPU: the
reference's own complex_scan golden vectors (float32: 1e-5 forward, 1e-4 gradients; bfloat16 b
with float32 a: the outputs in bfloat16 and the gradients against those outputs, 1e-2), the
float64 oracle at shapes with many chunks and mode blocks, dtype rules, error behaviour, and
size-independent properties at a config-3-like size (B=16, L=8192, 1024 modes): the scan is
linear in b, a prefix of the sequence gives the same prefix of the result, and the float32
last state agrees with the last output."""
import numpy as np
import pytest
import torch

from oracle import sparc_oracle as O

pytestmark = pytest.mark.gpu


def _t(a, dtype=torch.float32, grad=True):
    return torch.tensor(np.asarray(a), dtype=torch.float32, device="cuda").to(dtype).requires_grad_(grad)


def _rel(got, ref):
    return O.rel_l2(got.detach().double().cpu().numpy(), ref)


def test_complex_scan_matches_reference_golden(golden):
    from sparc_b200 import complex_scan, complex_scan_with_last

    d = golden("complex")
    t = [_t(d[k]) for k in ("ar", "ai", "br", "bi")]
    out_r, out_i = complex_scan(*t)
    assert out_r.dtype == torch.float32 and out_r.shape == t[0].shape
    assert _rel(out_r, d["f32_out_r"]) < 1e-5 and _rel(out_i, d["f32_out_i"]) < 1e-5
    gr, gi = _t(d["gr"], grad=False), _t(d["gi"], grad=False)
    ((out_r * gr).sum() + (out_i * gi).sum()).backward()
    for k, x in zip(("ar", "ai", "br", "bi"), t):
        assert x.grad.dtype == torch.float32
        assert _rel(x.grad, d["f32_grad_" + k]) < 1e-4, k
    o_r, o_i, l_r, l_i = complex_scan_with_last(*(x.detach() for x in t))
    assert torch.equal(o_r, out_r.detach()) and torch.equal(o_i, out_i.detach())
    assert l_r.dtype == torch.float32 and _rel(l_r, d["with_last_last_r"]) < 1e-5
    assert _rel(l_i, d["with_last_last_i"]) < 1e-5


def test_complex_scan_bf16_writes_golden(golden):
    """float32 a with bfloat16 b: outputs in bfloat16, every gradient computed in a's dtype
    against the bfloat16 outputs (cast to b's dtype for b by autograd)."""
    from sparc_b200 import complex_scan

    d = golden("complex")
    t = [_t(d["ar"]), _t(d["ai"]), _t(d["bf16b_br"], torch.bfloat16), _t(d["bf16b_bi"], torch.bfloat16)]
    out_r, out_i = complex_scan(*t)
    assert out_r.dtype == torch.bfloat16 and out_i.dtype == torch.bfloat16
    assert _rel(out_r, d["bf16b_out_r"]) < 1e-2 and _rel(out_i, d["bf16b_out_i"]) < 1e-2
    gr, gi = _t(d["gr"], grad=False), _t(d["gi"], grad=False)
    ((out_r.float() * gr).sum() + (out_i.float() * gi).sum()).backward()
    assert t[0].grad.dtype == torch.float32 and t[2].grad.dtype == torch.bfloat16
    for k, x in zip(("ar", "ai", "br", "bi"), t):
        assert _rel(x.grad, d["bf16b_grad_" + k]) < 1e-2, k


@pytest.mark.parametrize("B,L,M,adt,bdt", [(2, 300, 300, torch.float32, torch.float32),
                                           (3, 1000, 40, torch.float32, torch.float32),
                                           (1, 33, 1, torch.float32, torch.float32),
                                           (2, 257, 130, torch.bfloat16, torch.bfloat16),
                                           (2, 96, 64, torch.bfloat16, torch.float32)])
def test_complex_scan_matches_oracle(B, L, M, adt, bdt):
    """Many chunks (L = 1000: 32 chunks per row), ragged lengths, one mode, modes across 128-mode
    blocks, every dtype pairing; float32 1e-5 / 1e-4, bfloat16 2e-2."""
    from sparc_b200 import complex_scan

    rng = np.random.default_rng(B * L + M)
    rad = 0.95 + 0.05 * rng.random((B, L, M))
    ang = 0.5 * rng.standard_normal((B, L, M))
    ar, ai = rad * np.cos(ang), rad * np.sin(ang)
    br, bi = 0.5 * rng.standard_normal((B, L, M)), 0.5 * rng.standard_normal((B, L, M))
    gr, gi = rng.standard_normal((B, L, M)), rng.standard_normal((B, L, M))
    t = [_t(ar, adt), _t(ai, adt), _t(br, bdt), _t(bi, bdt)]
    out_r, out_i = complex_scan(*t)
    assert out_r.dtype == bdt
    # the oracle on the kernels' own inputs (rounded to their dtypes)
    a_in = [x.detach().double().cpu().numpy() for x in t]
    hr, hi, _, _ = O.complex_scan_forward(*a_in)
    low = torch.bfloat16 in (adt, bdt)
    ft, bt = (2e-2, 2e-2) if low else (1e-5, 1e-4)
    assert _rel(out_r, hr) < ft and _rel(out_i, hi) < ft
    g = [_t(gr, bdt, False), _t(gi, bdt, False)]
    ((out_r.float() * g[0].float()).sum() + (out_i.float() * g[1].float()).sum()).backward()
    yr, yi = out_r.detach().double().cpu().numpy(), out_i.detach().double().cpu().numpy()
    grads = O.complex_scan_backward(a_in[0], a_in[1], yr, yi, *(x.double().cpu().numpy() for x in g))
    for k, x, ref in zip(("ar", "ai", "br", "bi"), t, grads):
        assert _rel(x.grad, ref) < bt, k


def test_complex_scan_errors_and_cpu():
    from sparc_b200 import complex_scan, complex_scan_with_last

    a = torch.zeros(2, 8, 4, device="cuda")
    with pytest.raises(ValueError, match=r"complex scan expects matching \[B, L, M\] tensors"):
        complex_scan(a, a, a, a[:, :4])
    with pytest.raises(ValueError, match=r"complex scan expects matching \[B, L, M\] tensors"):
        complex_scan_with_last(a[0], a[0], a[0], a[0])
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        complex_scan(a.cpu(), a.cpu(), a.cpu(), a.cpu())


def test_complex_scan_properties_at_size():
    """B=16, L=8192, 1024 modes, float32: linear in b (scan(a, b1 + b2) = scan(a, b1) + scan(a,
    b2)), prefixes (the first 3000 tokens alone give the same first 3000 outputs), and the
    float32 last state equals the last output."""
    from sparc_b200 import complex_scan_with_last

    B, L, M = 16, 8192, 1024
    g = torch.Generator(device="cuda").manual_seed(3)
    rad = 0.999 + 0.001 * torch.rand(B, L, M, generator=g, device="cuda")
    ang = 0.1 * torch.randn(B, L, M, generator=g, device="cuda")
    ar, ai = rad * torch.cos(ang), rad * torch.sin(ang)
    del rad, ang
    b1r, b1i = torch.randn(B, L, M, generator=g, device="cuda"), torch.randn(B, L, M, generator=g, device="cuda")
    y1r, y1i, l1r, l1i = complex_scan_with_last(ar, ai, b1r, b1i)
    assert torch.equal(l1r, y1r[:, -1]) and torch.equal(l1i, y1i[:, -1])
    p = 3000
    pr, pi_, _, _ = complex_scan_with_last(ar[:, :p], ai[:, :p], b1r[:, :p], b1i[:, :p])
    scale = y1r[:, :p].abs().max()
    assert float((pr - y1r[:, :p]).abs().max() / scale) < 1e-5
    assert float((pi_ - y1i[:, :p]).abs().max() / scale) < 1e-5
    b2r, b2i = torch.randn(B, L, M, generator=g, device="cuda"), torch.randn(B, L, M, generator=g, device="cuda")
    y2r, y2i, _, _ = complex_scan_with_last(ar, ai, b2r, b2i)
    ysr, ysi, _, _ = complex_scan_with_last(ar, ai, b1r + b2r, b1i + b2i)
    ref = y1r + y2r
    assert float((ysr - ref).norm() / ref.norm()) < 1e-5
    assert float((ysi - (y1i + y2i)).norm() / (y1i + y2i).norm()) < 1e-5
