"""The scan-level entry points (sparc_b200.scan: sparc_scan, sparc_tiled_serial_scan,
sparc_chunk_scan, sparc_scan_with_last, sparc_training_scan_dispatch) on the GPU: the reference's
own sparc_tiled_serial_scan golden vectors (h0, segment resets, gradient of the last state;
float32: 1e-4 forward, 1e-3 gradients) and the float64 oracle's scan and adjoint for other
shapes (two and four CTAs of modes, bfloat16 writes at 2e-2), with controls inside the module
controller's range and far outside it (the scan-level functions take any eta and delta)."""
import numpy as np
import pytest
import torch

from oracle import sparc_oracle as O

pytestmark = pytest.mark.gpu


def _cuda(d, keys, grad=True):
    return {k: torch.tensor(d[k], dtype=torch.float32, device="cuda").requires_grad_(grad) for k in keys}


def test_tiled_serial_scan_matches_reference_golden(golden):
    from sparc_b200 import scan

    d = golden("tiled_h0_reset")
    t = _cuda(d, ("eta", "delta", "write_r", "write_i", "h0_r", "h0_i", "p_nu_log", "p_theta_log"))
    out_r, out_i, last_r, last_i = scan.sparc_tiled_serial_scan(
        t["eta"], t["delta"], t["p_nu_log"], t["p_theta_log"], t["write_r"], t["write_i"],
        segment_pos=torch.tensor(d["segment_pos"], device="cuda"), initial_state=(t["h0_r"], t["h0_i"]))
    for got, ref in ((out_r, "out_r"), (out_i, "out_i"), (last_r, "last_r"), (last_i, "last_i")):
        assert O.rel_l2(got.detach().double().cpu().numpy(), d[ref]) < 1e-4, ref
    g = {k: torch.tensor(d[k], device="cuda") for k in ("d_out_r", "d_out_i", "d_last_r", "d_last_i")}
    ((out_r.double() * g["d_out_r"]).sum() + (out_i.double() * g["d_out_i"]).sum()
     + (last_r.double() * g["d_last_r"]).sum() + (last_i.double() * g["d_last_i"]).sum()).backward()
    for k, ref in (("eta", "grad_eta"), ("delta", "grad_delta"), ("write_r", "grad_write_r"),
                   ("write_i", "grad_write_i"), ("h0_r", "grad_h0_r"), ("h0_i", "grad_h0_i"),
                   ("p_nu_log", "grad_nu_log"), ("p_theta_log", "grad_theta_log")):
        assert O.rel_l2(t[k].grad.double().cpu().numpy(), d[ref]) < 1e-3, k


def _problem(B, L, M, seed, wide=False):
    rng = np.random.default_rng(seed)
    p = rng.standard_normal((B, L, 2)) * 0.8
    eta, delta = np.log(16.0) * np.tanh(p[..., 1]), 0.5 * np.pi * np.tanh(p[..., 0])
    if wide:  # controls far outside the module controller's range: the scan takes any values
        eta = rng.uniform(-6.0, 4.0, (B, L))
        delta = rng.standard_normal((B, L)) * 6.0
    P = O.Params.from_mapping({"nu_log": rng.standard_normal(M) * 0.5 - 1.5, "theta_log": rng.standard_normal(M) * 0.5,
                               "phase_direction": np.zeros(2 * M + 1), "radial_direction": np.zeros(2 * M + 1),
                               "write_log_gain": np.zeros(M), "energy_response": np.zeros(M),
                               "write_phase_response": np.zeros(M), "write_radial_response": np.zeros(M)})
    br, bi = rng.standard_normal((B, L, M)) * 0.3, rng.standard_normal((B, L, M)) * 0.3
    gr, gi = rng.standard_normal((B, L, M)), rng.standard_normal((B, L, M))
    return eta, delta, P, br, bi, gr, gi


@pytest.mark.parametrize("wide", [False, True], ids=["module_range", "wide_controls"])
@pytest.mark.parametrize("B,L,M,dtype,tol", [(2, 50, 300, torch.float32, (1e-4, 1e-3)),
                                             (2, 64, 40, torch.bfloat16, (2e-2, 2e-2)),
                                             (3, 200, 1024, torch.float32, (1e-4, 1e-3))])
def test_sparc_scan_matches_oracle(B, L, M, dtype, tol, wide):
    """The scan against the float64 oracle, with controls inside the module controller's range
    (|eta| < ln16, |delta| < pi/2) and far outside it (eta in [-6, 4], delta ~ 6 N(0, 1))."""
    from sparc_b200 import scan

    eta, delta, P, br, bi, gr, gi = _problem(B, L, M, M, wide)
    dev = "cuda"
    te = torch.tensor(eta, dtype=torch.float32, device=dev, requires_grad=True)
    td = torch.tensor(delta, dtype=torch.float32, device=dev, requires_grad=True)
    tn = torch.tensor(P.nu_log, dtype=torch.float32, device=dev, requires_grad=True)
    tt = torch.tensor(P.theta_log, dtype=torch.float32, device=dev, requires_grad=True)
    tbr = torch.tensor(br, device=dev).to(dtype).requires_grad_(True)
    tbi = torch.tensor(bi, device=dev).to(dtype).requires_grad_(True)
    out_r, out_i = scan.sparc_scan(te, td, tn, tt, tbr, tbi)
    assert out_r.dtype == dtype and out_r.shape == (B, L, M) and out_r.is_contiguous() and out_i.is_contiguous()
    ar, ai, _, _ = O.transition(eta, delta, P)
    brd, bid = tbr.detach().double().cpu().numpy(), tbi.detach().double().cpu().numpy()
    hr, hi = O._scan(ar, ai, brd, bid)
    ft, bt = tol
    assert O.rel_l2(out_r.detach().double().cpu().numpy(), hr) < ft
    assert O.rel_l2(out_i.detach().double().cpu().numpy(), hi) < ft
    ((out_r.double() * torch.tensor(gr, device=dev)).sum() + (out_i.double() * torch.tensor(gi, device=dev)).sum()).backward()
    sc = O.scan_backward(eta, delta, P, hr, hi, gr, gi)
    for got, ref in ((tbr.grad, sc["lam_r"]), (tbi.grad, sc["lam_i"]), (te.grad, sc["eta"]), (td.grad, sc["delta"]),
                     (tn.grad, sc["nu_log"]), (tt.grad, sc["theta_log"])):
        assert O.rel_l2(got.double().cpu().numpy(), ref) < bt
    # the other entry points compute the same scan
    o_r, o_i, l_r, l_i = scan.sparc_scan_with_last(te, td, tn, tt, tbr, tbi)
    assert torch.equal(o_r, out_r.detach()) and torch.equal(o_i, out_i.detach())
    # (the last state is float32 and may come from the chunk carries: compare to rounding)
    assert O.rel_l2(l_r.double().cpu().numpy(), hr[:, -1]) < ft and O.rel_l2(l_i.double().cpu().numpy(), hi[:, -1]) < ft
    if L % 16 == 0:
        y = scan.sparc_training_scan_dispatch(te.detach(), td.detach(), tn.detach(), tt.detach(), tbr.detach(),
                                              tbi.detach(), chunk_size=16, fused_output_relu=True)
        assert torch.equal(y, torch.cat((out_r.detach(), out_i.detach()), -1).relu())
