"""The scan-level entry points (sparc_b200.scan) on CPU, with the projection-mode kernel call
(`scan._core`) replaced by a differentiable float64 restatement of what those kernels compute
(itself checked against the pinned oracle below): the change of variables, the plumbing, the
output layout and the gradients through it against the reference's own sparc_tiled_serial_scan
golden vectors (h0, segment resets, gradient of the last state), the routing of the dispatch,
the reference's argument checks, and that real inputs on CPU still fail (no CPU path). One test
goes through the real kernel call (scan._core and the projection-mode autograd function) with only
the two ctypes wrappers underneath emulated. The kernels themselves run in
tests/test_gpu_scan_functions.py."""
import math

import numpy as np
import pytest
import torch

from oracle import jax_layer_oracle as J
from oracle import sparc_oracle as O

LN16, HALF_PI = math.log(16.0), 0.5 * math.pi


def _standin_core(u, p, nu_log, theta_log, h0, reset):
    """What the projection-mode kernels compute for a linear content and zero write_log_gain /
    write responses, in float64 torch: tau = tanh(p), eta = ln16 tau1, delta = pi/2 tau0, the
    write gain sqrt(expm1(-2 nu e^eta) / expm1(-2 nu)) u, and the scan with h0 and resets."""
    dt = u.dtype
    u, p = u.double(), p.double()
    B, L, M2 = u.shape
    M = M2 // 2
    tau = torch.tanh(p)
    eta, delta = LN16 * tau[..., 1], HALF_PI * tau[..., 0]
    nu, theta = torch.exp(nu_log.double()), torch.exp(theta_log.double())
    z = nu * torch.exp(eta)[..., None]
    rho = torch.exp(-z)
    phi = theta + (1.0 - rho) * delta[..., None]
    ar, ai = rho * torch.cos(phi), rho * torch.sin(phi)
    if reset is not None:
        keep = (reset == 0).double()[..., None]
        ar, ai = ar * keep, ai * keep
    gain = torch.sqrt(torch.expm1(-2.0 * z) / torch.expm1(-2.0 * nu))
    br, bi = gain * u[..., :M], gain * u[..., M:]
    hr = torch.zeros(B, M, dtype=torch.float64) if h0 is None else h0[0].double()
    hi = torch.zeros(B, M, dtype=torch.float64) if h0 is None else h0[1].double()
    out = []
    for t in range(L):
        hr, hi = ar[:, t] * hr - ai[:, t] * hi + br[:, t], ai[:, t] * hr + ar[:, t] * hi + bi[:, t]
        out.append(torch.cat((hr, hi), -1))
    return torch.stack(out, 1).to(dt), hr.float(), hi.float()


@pytest.fixture
def standin(monkeypatch):
    from sparc_b200 import scan

    monkeypatch.setattr(scan, "_core", _standin_core)
    return scan


def _params(d):
    return O.Params.from_mapping({k[2:]: d[k] for k in d.files if k.startswith("p_")})


def test_standin_matches_the_oracle_projection_mode():
    """The stand-in is the oracle's projection-mode recurrence (the JAX layer's gain and the
    shared transition) with zero write_log_gain and responses and a linear content."""
    rng = np.random.default_rng(0)
    B, L, M = 2, 9, 5
    u = rng.standard_normal((B, L, 2 * M))
    p = rng.standard_normal((B, L, 2)) * 0.7
    P = O.Params.from_mapping({"nu_log": rng.standard_normal(M) * 0.5 - 1.0, "theta_log": rng.standard_normal(M) * 0.3,
                               "phase_direction": np.zeros(2 * M + 1), "radial_direction": np.zeros(2 * M + 1),
                               "write_log_gain": np.zeros(M), "energy_response": np.zeros(M),
                               "write_phase_response": np.zeros(M), "write_radial_response": np.zeros(M)})
    eta, delta = LN16 * np.tanh(p[..., 1]), HALF_PI * np.tanh(p[..., 0])
    ga = J._gain_terms(eta, delta, P)
    ar, ai, _, _ = O.transition(eta, delta, P)
    hr, hi = O._scan(ar, ai, ga["gain"] * u[..., :M], ga["gain"] * u[..., M:])
    h, lr, li = _standin_core(torch.tensor(u), torch.tensor(p), torch.tensor(P.nu_log), torch.tensor(P.theta_log),
                              None, None)
    assert O.rel_l2(h.numpy(), np.concatenate((hr, hi), -1)) < 1e-12


def test_tiled_serial_scan_matches_reference_golden(standin, golden):
    d = golden("tiled_h0_reset")
    t = {k: torch.tensor(d[k], dtype=torch.float32) for k in ("eta", "delta", "write_r", "write_i", "h0_r", "h0_i",
                                                              "p_nu_log", "p_theta_log")}
    for k in ("eta", "delta", "write_r", "write_i", "h0_r", "h0_i", "p_nu_log", "p_theta_log"):
        t[k].requires_grad_(True)
    out_r, out_i, last_r, last_i = standin.sparc_tiled_serial_scan(
        t["eta"], t["delta"], t["p_nu_log"], t["p_theta_log"], t["write_r"], t["write_i"],
        segment_pos=torch.tensor(d["segment_pos"]), initial_state=(t["h0_r"], t["h0_i"]))
    assert out_r.dtype == torch.float32 and out_r.is_contiguous() and last_r.shape == (2, 6)
    for got, ref in ((out_r, "out_r"), (out_i, "out_i"), (last_r, "last_r"), (last_i, "last_i")):
        assert O.rel_l2(got.detach().double().numpy(), d[ref]) < 1e-5, ref
    loss = ((out_r.double() * torch.tensor(d["d_out_r"])).sum() + (out_i.double() * torch.tensor(d["d_out_i"])).sum()
            + (last_r.double() * torch.tensor(d["d_last_r"])).sum() + (last_i.double() * torch.tensor(d["d_last_i"])).sum())
    loss.backward()
    for k, ref in (("eta", "grad_eta"), ("delta", "grad_delta"), ("write_r", "grad_write_r"),
                   ("write_i", "grad_write_i"), ("h0_r", "grad_h0_r"), ("h0_i", "grad_h0_i"),
                   ("p_nu_log", "grad_nu_log"), ("p_theta_log", "grad_theta_log")):
        assert O.rel_l2(t[k].grad.double().numpy(), d[ref]) < 1e-4, k


def test_scan_variants_agree(standin, golden):
    d = golden("tiled_h0_reset")
    eta, delta = torch.tensor(d["eta"]).float(), torch.tensor(d["delta"]).float()
    nl, tl = torch.tensor(d["p_nu_log"]).float(), torch.tensor(d["p_theta_log"]).float()
    br, bi = torch.tensor(d["write_r"]).float(), torch.tensor(d["write_i"]).float()
    ref_r, ref_i = standin.sparc_scan(eta, delta, nl, tl, br, bi)
    # the oracle's scan of the same controls and writes (no h0, no resets)
    ar, ai, _, _ = O.transition(d["eta"], d["delta"], _params(d))
    hr, hi = O._scan(ar, ai, d["write_r"], d["write_i"])
    assert O.rel_l2(ref_r.double().numpy(), hr) < 1e-5 and O.rel_l2(ref_i.double().numpy(), hi) < 1e-5
    o_r, o_i, l_r, l_i = standin.sparc_scan_with_last(eta, delta, nl, tl, br, bi)
    assert torch.equal(o_r, ref_r) and torch.equal(l_r, ref_r[:, -1]) and torch.equal(l_i, ref_i[:, -1])
    c_r, c_i = standin.sparc_chunk_scan(eta[:, :32], delta[:, :32], nl, tl, br[:, :32], bi[:, :32], chunk_size=32)
    assert torch.allclose(c_r, ref_r[:, :32], rtol=1e-6, atol=1e-7)
    y = standin.sparc_chunk_scan(eta[:, :32], delta[:, :32], nl, tl, br[:, :32], bi[:, :32], chunk_size=16,
                                 fused_output_relu=True)
    assert torch.allclose(y, torch.cat((ref_r[:, :32], ref_i[:, :32]), -1).relu(), rtol=1e-6, atol=1e-7)
    # the dispatch: a whole number of chunks goes to the chunked scan, a partial chunk, resets or
    # an initial state to the tiled serial scan; the results are the same scan
    dr, di = standin.sparc_training_scan_dispatch(eta[:, :32], delta[:, :32], nl, tl, br[:, :32], bi[:, :32])
    assert torch.allclose(dr, ref_r[:, :32], rtol=1e-6, atol=1e-7) and torch.allclose(di, ref_i[:, :32], rtol=1e-6, atol=1e-7)
    seg = torch.tensor(d["segment_pos"])
    tr, ti = standin.sparc_training_scan_dispatch(eta, delta, nl, tl, br, bi, segment_pos=seg)
    s_r, s_i, _, _ = standin.sparc_tiled_serial_scan(eta, delta, nl, tl, br, bi, segment_pos=seg)
    assert torch.equal(tr, s_r) and torch.equal(ti, s_i)


def test_fused_write(standin, golden):
    """raw_x times sqrt(1 - e^{-2 nu}) + 1e-8 as the writes, the gradient reaching raw_x."""
    d = golden("tiled_h0_reset")
    eta, delta = torch.tensor(d["eta"]).float()[:, :32], torch.tensor(d["delta"]).float()[:, :32]
    nl, tl = torch.tensor(d["p_nu_log"]).float(), torch.tensor(d["p_theta_log"]).float()
    raw = torch.tensor(d["x"]).float()[:, :32].requires_grad_(True)
    out_r, out_i = standin.sparc_chunk_scan(eta, delta, nl, tl, None, None, chunk_size=16, raw_x=raw, fused_write=True)
    gamma = torch.sqrt(1.0 - torch.exp(-2.0 * torch.exp(nl))) + 1e-8
    ref_r, ref_i = standin.sparc_scan(eta, delta, nl, tl, raw[..., :6].detach() * gamma, raw[..., 6:].detach() * gamma)
    assert torch.allclose(out_r, ref_r, rtol=1e-6, atol=1e-7) and torch.allclose(out_i, ref_i, rtol=1e-6, atol=1e-7)
    (out_r.sum() + out_i.sum()).backward()
    assert raw.grad is not None and raw.grad.shape == raw.shape and bool(raw.grad.abs().sum() > 0)


def test_reference_argument_checks():
    from sparc_b200 import scan

    e, dl = torch.zeros(2, 32), torch.zeros(2, 32)
    nl, tl = torch.zeros(4), torch.zeros(4)
    b = torch.zeros(2, 32, 4)
    with pytest.raises(ValueError, match="controls must be matching"):
        scan.sparc_scan(e, dl[:, :16], nl, tl, b, b)
    with pytest.raises(ValueError, match="writes must be matching"):
        scan.sparc_scan(e, dl, nl, tl, b, b[..., :3])
    with pytest.raises(ValueError, match="disagree"):
        scan.sparc_scan(e, dl, nl[:3], tl, b, b)
    with pytest.raises(ValueError, match="block_size"):
        scan.sparc_tiled_serial_scan(e, dl, nl, tl, b, b, block_size=48)
    with pytest.raises(ValueError, match="segment_pos"):
        scan.sparc_tiled_serial_scan(e, dl, nl, tl, b, b, segment_pos=torch.ones(2, 31))
    with pytest.raises(ValueError, match="initial SPARC states"):
        scan.sparc_tiled_serial_scan(e, dl, nl, tl, b, b, initial_state=(torch.zeros(2, 3), torch.zeros(2, 3)))
    with pytest.raises(ValueError, match="chunk size"):
        scan.sparc_chunk_scan(e, dl, nl, tl, b, b, chunk_size=24)
    with pytest.raises(ValueError, match="mode block size"):
        scan.sparc_chunk_scan(e, dl, nl, tl, b, b, mode_block_size=100)
    with pytest.raises(ValueError, match="raw_x is required"):
        scan.sparc_training_scan_dispatch(e, dl, nl, tl, b, b, fused_write=True)
    with pytest.raises(ValueError, match="raw_x"):
        scan.sparc_chunk_scan(e, dl, nl, tl, None, None, raw_x=torch.zeros(2, 32, 7), fused_write=True)
    with pytest.raises(NotImplementedError, match="controller_backward_cache"):
        scan.sparc_chunk_scan(e, dl, nl, tl, b, b, controller_backward_cache=(e,) * 6)
    with pytest.raises(RuntimeError, match="CUDA"):  # well-formed CPU inputs: there is no CPU path
        scan.sparc_scan(e, dl, nl, tl, b, b)


class _EmuSaved:
    pass


def _emu_core_forward(u, p, modal, h0, reset, lin, max_spin):
    """Stands in for projection._core_forward (the sparc_mixer_forward call in projection mode)
    with the float64 restatement, keeping its autograd graph for _emu_core_backward."""
    nu_log, theta_log, wlg, wpr, wrr = modal
    assert lin and not any(bool(t.abs().sum()) for t in (wlg, wpr, wrr))  # what the scan entry points pass
    sv = _EmuSaved()
    sv.leaves = [t.detach().double().requires_grad_(True) for t in (u, p, nu_log, theta_log)]
    sv.h0 = None if h0 is None else [t.detach().double().requires_grad_(True) for t in h0]
    sv.u_dtype = u.dtype
    with torch.enable_grad():
        sv.out = _standin_core(sv.leaves[0], sv.leaves[1], sv.leaves[2], sv.leaves[3], sv.h0, reset)
    h, lr, li = sv.out
    return h.detach().to(u.dtype), lr.detach(), li.detach(), sv


def _emu_core_backward(sv, dh, dlast_r, dlast_i):
    """Stands in for projection._core_backward: (du, dp, five modal gradients, gh0 or None)."""
    h, lr, li = sv.out
    gouts = [torch.zeros_like(h) if dh is None else dh.double(), torch.zeros_like(lr) if dlast_r is None else dlast_r,
             torch.zeros_like(li) if dlast_i is None else dlast_i]
    ins = sv.leaves + (sv.h0 or [])
    gr = torch.autograd.grad([h, lr, li], ins, gouts, allow_unused=True)
    gr = [torch.zeros_like(x) if g is None else g for g, x in zip(gr, ins)]
    du, dp, dnu, dth = gr[0].to(sv.u_dtype), gr[1].float(), gr[2].float(), gr[3].float()
    zeros = torch.zeros_like(dnu)
    gh0 = None if sv.h0 is None else (gr[4].float(), gr[5].float())
    return du, dp, [dnu, dth, zeros, zeros, zeros], gh0


def test_real_core_call_with_emulated_kernels(monkeypatch, golden):
    """The scan entry points through their real kernel call (scan._core -> the projection-mode
    autograd function), with only the two ctypes wrappers underneath emulated: the argument
    order, the zero write parameters, h0 / resets and the gradients' way back, against the
    reference's golden vectors."""
    from sparc_b200 import _lib, projection, scan

    monkeypatch.setattr(projection, "_core_forward", _emu_core_forward)
    monkeypatch.setattr(projection, "_core_backward", _emu_core_backward)
    monkeypatch.setattr(_lib, "require_cuda", lambda t, name: None)
    d = golden("tiled_h0_reset")
    t = {k: torch.tensor(d[k], dtype=torch.float32).requires_grad_(True)
         for k in ("eta", "delta", "write_r", "write_i", "h0_r", "h0_i", "p_nu_log", "p_theta_log")}
    out_r, out_i, last_r, last_i = scan.sparc_tiled_serial_scan(
        t["eta"], t["delta"], t["p_nu_log"], t["p_theta_log"], t["write_r"], t["write_i"],
        segment_pos=torch.tensor(d["segment_pos"]), initial_state=(t["h0_r"], t["h0_i"]))
    for got, ref in ((out_r, "out_r"), (out_i, "out_i"), (last_r, "last_r"), (last_i, "last_i")):
        assert O.rel_l2(got.detach().double().numpy(), d[ref]) < 1e-5, ref
    ((out_r.double() * torch.tensor(d["d_out_r"])).sum() + (out_i.double() * torch.tensor(d["d_out_i"])).sum()
     + (last_r.double() * torch.tensor(d["d_last_r"])).sum() + (last_i.double() * torch.tensor(d["d_last_i"])).sum()
     ).backward()
    for k, ref in (("eta", "grad_eta"), ("delta", "grad_delta"), ("write_r", "grad_write_r"),
                   ("write_i", "grad_write_i"), ("h0_r", "grad_h0_r"), ("h0_i", "grad_h0_i"),
                   ("p_nu_log", "grad_nu_log"), ("p_theta_log", "grad_theta_log")):
        assert O.rel_l2(t[k].grad.double().numpy(), d[ref]) < 1e-4, k


def test_module_level_aliases(standin, golden):
    import sparc_b200

    d = golden("tiled_h0_reset")
    args = [torch.tensor(d[k]).float() for k in ("eta", "delta", "p_nu_log", "p_theta_log", "write_r", "write_i")]
    a, b = standin.sparc_scan_precomputed_decay(*args), standin.sparc_scan(*args)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    m = sparc_b200.SPARCMixer(8)
    with pytest.raises(ValueError, match="batch, length, 8"):
        sparc_b200.run_sequence(m, torch.randn(2, 3, 6))
    with pytest.raises(RuntimeError, match="CUDA"):
        sparc_b200.run_sequence(m, torch.randn(2, 3, 8), True)
    sparc_b200.prepare_decode(m)
    assert m._inference_fused
    with pytest.raises(RuntimeError, match="CUDA"):
        sparc_b200.run_decode_step(m, torch.randn(2, 8), (torch.zeros(2, 4), torch.zeros(2, 4)), None)


def test_controls_at_and_beyond_the_bound(standin):
    """eta at or beyond ln16 (delta beyond pi/2) is clamped to just inside the bound: finite
    states and gradients, the writes kept exactly, the transition of the clamped controls."""
    B, L, M = 1, 6, 3
    eta = torch.tensor([[LN16, -LN16, 5.0, 0.3, -9.0, 0.0]], requires_grad=True)
    delta = torch.tensor([[HALF_PI, 2.0, -HALF_PI, 0.1, 0.0, -3.0]], requires_grad=True)
    nl, tl = torch.full((M,), -1.0), torch.full((M,), 0.2)
    br, bi = torch.randn(B, L, M), torch.randn(B, L, M)
    out_r, out_i = standin.sparc_scan(eta, delta, nl, tl, br, bi)
    assert bool(torch.isfinite(out_r).all()) and bool(torch.isfinite(out_i).all())
    edge = 1.0 - 2.0 ** -23
    ec = (eta.detach().double() / LN16).clamp(-edge, edge) * LN16
    dc = (delta.detach().double() / HALF_PI).clamp(-edge, edge) * HALF_PI
    P = O.Params.from_mapping({"nu_log": nl.double().numpy(), "theta_log": tl.double().numpy()} | {
        k: np.zeros(2 * M + 1 if "direction" in k else M) for k in ("phase_direction", "radial_direction",
                                                                    "write_log_gain", "energy_response",
                                                                    "write_phase_response", "write_radial_response")})
    ar, ai, _, _ = O.transition(ec.numpy(), dc.numpy(), P)
    hr, hi = O._scan(ar, ai, br.double().numpy(), bi.double().numpy())
    assert O.rel_l2(out_r.detach().double().numpy(), hr) < 1e-5 and O.rel_l2(out_i.detach().double().numpy(), hi) < 1e-5
    (out_r.sum() + out_i.sum()).backward()
    assert bool(torch.isfinite(eta.grad).all()) and bool(torch.isfinite(delta.grad).all())
    assert float(eta.grad[0, 2]) == 0.0 and float(delta.grad[0, 5]) == 0.0  # clamped: no gradient
