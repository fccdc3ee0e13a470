"""GPU parity of the RTRL cell (rtrl_step_kernel / rtrl_grad_kernel) against the float64 oracle
(oracle/jax_layer_oracle.py: rtrl_step, rtrl_grads), over several steps with resets.

Tolerances (relative l2 against float64, per tensor): states and traces 1e-4 (float32
recurrence, like the forward bound); gradients 1e-3."""
import numpy as np
import pytest
import torch

from oracle import jax_layer_oracle as J
from oracle import sparc_oracle as O

pytestmark = pytest.mark.gpu


def _cell(W, M, seed, **kw):
    import sparc_b200

    torch.manual_seed(seed)
    cell = sparc_b200.SPARCRTRLCell(W, M, r_min=0.4, r_max=0.99, **kw).cuda()
    gen = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        cell.phase_controller.copy_(torch.randn(W + 1, generator=gen) * 0.8 / W ** 0.5)
        cell.retention_controller.copy_(torch.randn(W + 1, generator=gen) * 0.8 / W ** 0.5)
        cell.write_phase_response.copy_(torch.randn(M, generator=gen) * 0.5)
        cell.write_retention_response.copy_(torch.randn(M, generator=gen) * 0.5)
    params = {n: p.detach().double().cpu().numpy() for n, p in cell.named_parameters()}
    return cell, params


def _np(t):
    return t.detach().cpu().numpy().astype(np.complex128) if t.is_complex() else t.detach().double().cpu().numpy()


def _ri(a):
    """A complex array as real (re, im) pairs, for the relative-error helpers."""
    a = np.asarray(a)
    return np.stack((a.real, a.imag), axis=-1)


@pytest.mark.parametrize("B,W,M,act,out", [(4, 64, 64, "tanh", "relu"),     # the reference example's sizes
                                           (3, 40, 300, "linear", "linear"),  # three CTAs of modes
                                           (2, 5, 7, "tanh", "relu")])
def test_rtrl_steps_and_grads_match_oracle(B, W, M, act, out):
    import sparc_b200

    cell, params = _cell(W, M, 0, content_activation=act, output_activation=out)
    gen = torch.Generator(device="cuda").manual_seed(0)
    carry = cell.initial_carry(B)
    ref_state = np.zeros((B, M), np.complex128)
    ref_tr = J.init_traces(B, W, M)
    steps = 5
    for t in range(steps):
        x = torch.randn(B, W, generator=gen, device="cuda")
        reset = torch.zeros(B, dtype=torch.bool, device="cuda")
        if t == 3:
            reset[0] = True
        xg = x.clone().requires_grad_(True)
        prev_state = ref_state
        carry_new, y = cell(carry, xg, reset)
        ref_state, ref_tr = J.rtrl_step(params, prev_state, ref_tr, _np(x), _np(reset).astype(bool), act)
        assert O.rel_l2(_ri(_np(carry_new[0])), _ri(ref_state)) < 1e-4, f"step {t} state"
        for n in J.LAYER_NAMES[:9]:
            assert O.rel_l2(_ri(_np(carry_new[1][n])), _ri(ref_tr[n])) < 1e-4, f"step {t} trace {n}"
        # a loss on this step's output: gradients from the new traces plus the one-step input gradient
        w = torch.randn(B, 2 * M, generator=gen, device="cuda")
        cell.zero_grad(set_to_none=True)
        (y * w).sum().backward()
        s = ref_state
        wn = _np(w)
        mask_r = (s.real > 0) if out == "relu" else np.ones_like(s.real, bool)
        mask_i = (s.imag > 0) if out == "relu" else np.ones_like(s.imag, bool)
        g = J.rtrl_grads(params, prev_state, ref_tr, _np(x), wn[:, :M] * mask_r, wn[:, M:] * mask_i,
                         _np(reset).astype(bool), act)
        for n, p in cell.named_parameters():
            assert O.rel_l2(_np(p.grad), g[n]) < 1e-3, f"step {t} grad {n}"
        assert O.rel_l2(_np(xg.grad), g["x"]) < 1e-3, f"step {t} grad x"
        carry = carry_new
    assert isinstance(sparc_b200.SPARCRTRLCell, type)


def test_rtrl_carry_is_detached_and_api():
    import sparc_b200

    cell, _ = _cell(6, 4, 1)
    carry = cell.initial_carry(2)
    assert carry[0].shape == (2, 4) and carry[0].dtype == torch.complex64
    assert set(carry[1]) == set(J.LAYER_NAMES[:9])
    assert carry[1]["content_real"].shape == (2, 6, 4) and carry[1]["phase_controller"].shape == (2, 7, 4)
    nxt, y = cell(carry, torch.randn(2, 6, device="cuda"))
    assert y.shape == (2, 8) and y.requires_grad
    assert not nxt[0].requires_grad and not any(t.requires_grad for t in nxt[1].values())
    with pytest.raises(ValueError):
        cell(carry, torch.randn(2, 5, device="cuda"))
    with pytest.raises(ValueError):
        sparc_b200.SPARCRTRLCell(6, 4, output_activation="tanh")
