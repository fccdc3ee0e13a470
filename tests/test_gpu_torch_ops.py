"""The TORCH_LIBRARY operators (torch.ops.sparc_b200.*) give the same results as the module path
over the same C ABI (same kernels: bitwise equal for the mixer and decode, to rounding for the
real scan, whose lookback order can vary run to run)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

PARAMS = ("nu_log", "theta_log", "phase_direction", "radial_direction", "write_log_gain",
          "write_phase_response", "write_radial_response")


def test_mixer_and_decode_ops_match_module():
    import sparc_b200
    from sparc_b200 import torch_ops

    ops = torch_ops.load()
    torch.manual_seed(0)
    m = sparc_b200.SPARCMixer(64).cuda()
    with torch.no_grad():
        m.phase_direction.normal_(0, 0.15)
        m.radial_direction.normal_(0, 0.15)
    x = torch.randn(2, 70, 64, device="cuda", requires_grad=True)
    g = torch.randn(2, 70, 64, device="cuda")
    y, cache = m(x, return_cache=True)
    y.backward(g)
    p = [getattr(m, n).detach() for n in PARAMS]
    y2, lr, li, carry, controls, states = ops.mixer_forward(x.detach(), *p)
    assert torch.equal(y2, y.detach()) and torch.equal(lr, cache[0]) and torch.equal(li, cache[1])
    grads = ops.mixer_backward(x.detach(), y2, g, *p, carry, controls, states)
    assert torch.equal(grads[0], x.grad)
    names = ("nu_log", "theta_log", "phase_direction", "radial_direction", "write_log_gain",
             "energy_response", "write_phase_response", "write_radial_response")
    for n, t in zip(names, grads[1:]):
        assert torch.equal(t, getattr(m, n).grad), n
    # without the saved states the gradient kernel replays them: the same gradients to rounding
    replayed = ops.mixer_backward(x.detach(), y2, g, *p, carry, controls)
    for t, r in zip(grads, replayed):
        assert torch.allclose(r, t, rtol=1e-4, atol=1e-5)
    st = (torch.zeros(2, 32, device="cuda"), torch.zeros(2, 32, device="cuda"))
    m.prepare_inference()  # the fused decode kernel, which decode_step registers
    yd, sd = m.step(x.detach()[:, 0], st, None)
    yd2, nr, ni = ops.decode_step(x.detach()[:, 0].contiguous(), st[0], st[1], *p)
    assert torch.equal(yd2, yd) and torch.equal(nr, sd[0]) and torch.equal(ni, sd[1])


def test_real_scan_ops_match_module():
    import sparc_b200
    from sparc_b200 import torch_ops

    ops = torch_ops.load()
    a = (torch.rand(2, 64, 96, device="cuda") * 0.5 + 0.45).requires_grad_(True)
    b = torch.randn(2, 64, 96, device="cuda", requires_grad=True)
    g = torch.randn(2, 64, 96, device="cuda")
    out = sparc_b200.real_scan(a, b)
    out.backward(g)
    out2, carry, last = ops.real_scan_forward(a.detach(), b.detach())
    # (the real scan's decoupled lookback may compose its carries in another order run to run)
    assert torch.allclose(out2, out.detach(), rtol=1e-6, atol=1e-6)
    ga, gb = ops.real_scan_backward(a.detach(), b.detach(), g, carry)
    assert torch.allclose(ga, a.grad, rtol=1e-6, atol=1e-6) and torch.allclose(gb, b.grad, rtol=1e-6, atol=1e-6)


def test_operator_autograd_matches_module():
    """torch.ops.sparc_b200.mixer_forward / real_scan_forward are differentiable through their
    registered formulas: the same gradients as the module path (same kernels)."""
    import sparc_b200
    from sparc_b200 import torch_ops

    ops = torch_ops.load()
    torch.manual_seed(1)
    m = sparc_b200.SPARCMixer(48).cuda()
    with torch.no_grad():
        m.phase_direction.normal_(0, 0.15)
        m.radial_direction.normal_(0, 0.15)
    x = torch.randn(2, 41, 48, device="cuda", requires_grad=True)
    g = torch.randn(2, 41, 48, device="cuda")
    y, _ = m(x)
    y.backward(g)
    x2 = x.detach().clone().requires_grad_(True)
    p = [getattr(m, n).detach().clone().requires_grad_(True) for n in PARAMS]
    y2 = ops.mixer_forward(x2, *p)[0]
    y2.backward(g)
    assert torch.equal(y2.detach(), y.detach()) and torch.equal(x2.grad, x.grad)
    for n, t in zip(PARAMS, p):
        assert torch.equal(t.grad, getattr(m, n).grad), n
    a = (torch.rand(2, 50, 33, device="cuda") * 0.5 + 0.45).requires_grad_(True)
    b = torch.randn(2, 50, 33, device="cuda", requires_grad=True)
    gr = torch.randn(2, 50, 33, device="cuda")
    ga_, gb_ = torch.autograd.grad(sparc_b200.real_scan(a, b), (a, b), gr)
    a2 = a.detach().clone().requires_grad_(True)
    b2 = b.detach().clone().requires_grad_(True)
    ga2, gb2 = torch.autograd.grad(ops.real_scan_forward(a2, b2)[0], (a2, b2), gr)
    assert torch.allclose(ga2, ga_, rtol=1e-6, atol=1e-6) and torch.allclose(gb2, gb_, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("dtype,W,T", [(torch.float32, 512, 37), (torch.float32, 1024, 100),
                                       (torch.bfloat16, 2048, 70), (torch.bfloat16, 512, 49)])
def test_saved_state_and_replaying_gradient_kernels_agree(dtype, W, T):
    """The gradient kernel that reads the forward's saved states (halves in a two-stage ring
    without a cluster, whole tiles with the cluster's sums pushed between CTAs at W >= 1024) and
    the one that replays the states from the chunk carries give the same gradients (float32 to
    1e-4; bfloat16, whose replayed and saved states are both rounded to bfloat16, to 1e-2),
    with ragged last chunks."""
    from sparc_b200 import torch_ops

    ops = torch_ops.load()
    torch.manual_seed(1)
    p = [torch.randn(W // 2, device="cuda") * 0.3 - 1.0, torch.randn(W // 2, device="cuda") * 0.3,
         torch.randn(W + 1, device="cuda") / W ** 0.5, torch.randn(W + 1, device="cuda") / W ** 0.5,
         torch.randn(W // 2, device="cuda") * 0.1, torch.randn(W // 2, device="cuda") * 0.5,
         torch.randn(W // 2, device="cuda") * 0.5]
    x = torch.randn(3, T, W, device="cuda").to(dtype)
    g = torch.randn(3, T, W, device="cuda").to(dtype)
    y, lr, li, carry, controls, states = ops.mixer_forward(x, *p)
    saved = ops.mixer_backward(x, y, g, *p, carry, controls, states)
    replayed = ops.mixer_backward(x, y, g, *p, carry, controls)
    tol = 1e-4 if dtype == torch.float32 else 1e-2
    for k, (s, r) in enumerate(zip(saved, replayed)):
        s, r = s.double(), r.double()
        err = ((s - r).norm() / r.norm().clamp_min(1e-30)).item()
        assert err < tol, (k, err)
