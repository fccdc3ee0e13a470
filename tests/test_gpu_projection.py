"""GPU parity of the projection variant (the JAX sequence layer of sparc-impl as a torch module,
recurrence in libsparc_b200's projection mode) against the float64 oracle
(oracle/jax_layer_oracle.py).

Tolerances (relative l2 against float64, per tensor): float32 forward 1e-4, backward 1e-3;
bfloat16 activations 2e-2 (the same bounds as the mixer)."""
import numpy as np
import pytest
import torch

from oracle import jax_layer_oracle as J
from oracle import sparc_oracle as O

pytestmark = pytest.mark.gpu


def _layer(W, M, seed, act="tanh"):
    import sparc_b200

    torch.manual_seed(seed)
    m = sparc_b200.SPARCSequenceLayer(W, M, content_activation=act).cuda()
    gen = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():  # non-trivial controllers and gate responses
        m.phase_controller.copy_(torch.randn(W + 1, generator=gen) * 1.2 / W ** 0.5)
        m.retention_controller.copy_(torch.randn(W + 1, generator=gen) * 1.2 / W ** 0.5)
        m.write_phase_response.copy_(torch.randn(M, generator=gen) * 0.8)
        m.write_retention_response.copy_(torch.randn(M, generator=gen) * 0.8)
    params = {n: p.detach().double().cpu().numpy() for n, p in m.named_parameters()}
    return m, params


def _run(m, x, dy, **kw):
    x = x.clone().requires_grad_(True)
    out = m(x, **kw)
    y, last = out if isinstance(out, tuple) else (out, None)
    (y.double() * dy.double()).sum().backward()
    grads = {n: p.grad.double().cpu().numpy() for n, p in m.named_parameters()}
    grads["x"] = x.grad.double().cpu().numpy()
    return y.detach().double().cpu().numpy(), grads


def _check(y, g, y_ref, g_ref, fwd_tol, bwd_tol, label):
    e = O.rel_l2(y, y_ref)
    assert e < fwd_tol, f"{label} y rel-l2 {e:.3e}"
    for k in ("x",) + J.LAYER_NAMES:
        e = O.rel_l2(g[k], g_ref[k])
        assert e < bwd_tol, f"{label} grad {k} rel-l2 {e:.3e} (tol {bwd_tol})"


@pytest.mark.parametrize("B,T,W,M", [(2, 256, 64, 64),     # config 1 (JAX layer, d_model 64, 64 modes)
                                     (3, 100, 48, 37),     # odd modes, ragged chunk
                                     (2, 70, 40, 300),     # two CTAs of modes, W != 2M
                                     (1, 1, 8, 5)])
@pytest.mark.parametrize("act", ["tanh", "linear"])
def test_layer_matches_oracle_fp32(B, T, W, M, act):
    m, params = _layer(W, M, 0, act)
    gen = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(B, T, W, generator=gen, device="cuda")
    dy = torch.randn(B, T, W, generator=gen, device="cuda")
    y, g = _run(m, x, dy)
    xd, dyd = x.double().cpu().numpy(), dy.double().cpu().numpy()
    y_ref, _, _ = J.layer_forward(xd, params, content_activation=act)
    g_ref = J.layer_backward(xd, params, dyd, content_activation=act)
    _check(y, g, y_ref, g_ref, 1e-4, 1e-3, f"fp32 {B}x{T}x{W} M={M} {act}")


@pytest.mark.parametrize("B,T,W,M", [(2, 200, 128, 96),   # tensor-core products (W, 2M multiples of 8)
                                     (2, 130, 44, 29)])   # 2M = 58: torch products
def test_layer_matches_oracle_bf16(B, T, W, M):
    m, params = _layer(W, M, 1)
    gen = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(B, T, W, generator=gen, device="cuda").bfloat16()
    dy = torch.randn(B, T, W, generator=gen, device="cuda").bfloat16()
    y, g = _run(m, x, dy)
    xd, dyd = x.double().cpu().numpy(), dy.double().cpu().numpy()
    y_ref, _, _ = J.layer_forward(xd, params)
    g_ref = J.layer_backward(xd, params, dyd)
    _check(y, g, y_ref, g_ref, 2e-2, 2e-2, "bf16")


@pytest.mark.parametrize("dtype,tol", [(torch.float32, (1e-4, 1e-3)), (torch.bfloat16, (2e-2, 2e-2))])
def test_layer_state_and_resets(dtype, tol):
    """Initial state (with its gradient), segment resets and the returned last state (bfloat16:
    the tensor-core products)."""
    B, T, W, M = 2, 90, 32, 20
    m, params = _layer(W, M, 2)
    gen = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(B, T, W, generator=gen, device="cuda").to(dtype)
    dy = torch.randn(B, T, W, generator=gen, device="cuda").to(dtype)
    h0 = [torch.randn(B, M, generator=gen, device="cuda").requires_grad_(True) for _ in range(2)]
    pos = torch.arange(T, device="cuda").repeat(B, 1)
    pos[0, 40:] -= 40
    pos[1, 7:] -= 7
    xg = x.clone().requires_grad_(True)
    y, last = m(xg, state=(h0[0], h0[1]), segment_pos=pos, return_cache=True)
    dl = [torch.randn(B, M, generator=gen, device="cuda") for _ in range(2)]
    ((y.double() * dy.double()).sum() + (last[0] * dl[0]).sum() + (last[1] * dl[1]).sum()).backward()
    reset = (pos == 0).cpu().numpy()
    xd = x.double().cpu().numpy()
    h0d = (h0[0].detach().double().cpu().numpy(), h0[1].detach().double().cpu().numpy())
    dld = (dl[0].double().cpu().numpy(), dl[1].double().cpu().numpy())
    y_ref, last_ref, _ = J.layer_forward(xd, params, h0=h0d, reset=reset)
    g_ref = J.layer_backward(xd, params, dy.double().cpu().numpy(), h0=h0d, grad_last=dld, reset=reset)
    ft, bt = tol
    assert O.rel_l2(y.detach().double().cpu().numpy(), y_ref) < ft
    assert O.rel_l2(last[0].detach().double().cpu().numpy(), last_ref[0]) < ft
    assert O.rel_l2(xg.grad.double().cpu().numpy(), g_ref["x"]) < bt
    assert O.rel_l2(h0[0].grad.double().cpu().numpy(), g_ref["h0_r"]) < bt
    assert O.rel_l2(h0[1].grad.double().cpu().numpy(), g_ref["h0_i"]) < bt
    for n, p in m.named_parameters():
        assert O.rel_l2(p.grad.double().cpu().numpy(), g_ref[n]) < bt, n


def test_selection_layer_equals_mixer():
    """Under the selection parameters the projection path computes the torch mixer's states:
    relu of the layer is SPARCMixer's output from the same parameters (both on the GPU)."""
    import sparc_b200

    W = 64
    torch.manual_seed(3)
    mixer = sparc_b200.SPARCMixer(W).cuda()
    with torch.no_grad():
        mixer.phase_direction.copy_(torch.randn(W + 1) * 0.15)
        mixer.radial_direction.copy_(torch.randn(W + 1) * 0.15)
    P = O.Params.from_mapping({k: getattr(mixer, k).detach().double().cpu().numpy() for k in O.PARAM_NAMES})
    sel = J.selection_params(P)
    layer = sparc_b200.SPARCSequenceLayer(W, W // 2).cuda()
    with torch.no_grad():
        for n, p in layer.named_parameters():
            p.copy_(torch.as_tensor(sel[n], dtype=torch.float32))
    x = torch.randn(4, 300, W, device="cuda")
    with torch.no_grad():
        y_mixer, _ = mixer(x)
        y_layer = layer(x)
    assert O.rel_l2(torch.relu(y_layer).double().cpu().numpy(), y_mixer.double().cpu().numpy()) < 1e-5


def test_layer_api():
    import sparc_b200

    layer = sparc_b200.SPARCSequenceLayer(16, 8).cuda()
    names = {n for n, _ in layer.named_parameters()}
    assert names == set(J.LAYER_NAMES)
    assert tuple(layer.content_real.shape) == (16, 8) and tuple(layer.phase_controller.shape) == (17,)
    with pytest.raises(ValueError):
        layer(torch.randn(2, 5, 12, device="cuda"))
    with pytest.raises(ValueError):
        sparc_b200.SPARCSequenceLayer(16, 8, content_activation="relu")
