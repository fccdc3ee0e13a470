"""The scan-level entry points (sparc_b200.scan) on CPU, through their real Python path and the
real ctypes argument structs, with only the library underneath replaced by a fake that reads
those structs from host memory and computes what the kernels' scan-level mode computes with the
float64 oracle (transition, scan with h0 and resets, and its adjoint): the argument order,
`content_linear = 2`, the controls as (delta, eta) pairs, the writes as [b_r | b_i] rows, the
separate real and imaginary outputs (`y_im`), the controls the forward saves for the backward,
and the gradients' way back, against the reference's own sparc_tiled_serial_scan golden vectors
(h0, segment resets, gradient of the last state); controls far outside the module's controller
range pass through unchanged; the dispatch's routing; the reference's argument checks; and that
real inputs on CPU still fail (no CPU path). The kernels themselves run in
tests/test_gpu_scan_functions.py."""
import ctypes
import math

import numpy as np
import pytest
import torch

from oracle import sparc_oracle as O

LN16, HALF_PI = math.log(16.0), 0.5 * math.pi


def _arr(ptr, shape, dtype=np.float32):
    """A numpy view of host memory at `ptr`."""
    n = int(np.prod(shape))
    ct = {np.float32: ctypes.c_float, np.uint8: ctypes.c_uint8}[dtype]
    return np.ctypeslib.as_array((ct * n).from_address(ptr)).reshape(shape)


def _params(nl, tl, M):
    z = np.zeros(M)
    return O.Params.from_mapping({"nu_log": nl, "theta_log": tl, "phase_direction": np.zeros(2 * M + 1),
                                  "radial_direction": np.zeros(2 * M + 1), "write_log_gain": z,
                                  "energy_response": z, "write_phase_response": z, "write_radial_response": z})


class FakeLib:
    """The library's scan-level mode restated on host memory (float32 arrays only)."""

    def __init__(self):
        self.calls = []

    def sparc_mixer_carry_chunks(self, T, dt):
        return (T + 7) // 8

    def sparc_mixer_controls_floats(self):
        return 16

    def sparc_mixer_workspace_bytes(self, B, T, W, dt):
        return 1 << 10

    def sparc_last_error(self):
        return b""

    def sparc_mixer_forward(self, ref, stream):
        a = ref._obj
        self.calls.append(("forward", a.content_linear))
        assert a.content_linear == 2 and a.projections and a.y_im and a.dtype == 0
        assert not a.phase_direction and not a.radial_direction and not a.norm_weight
        B, T, W = a.batch, a.length, a.width
        M = W // 2
        u = _arr(a.x, (B, T, W)).astype(np.float64)
        pr = _arr(a.projections, (B, T, 2)).astype(np.float64)
        delta, eta = pr[..., 0], pr[..., 1]
        P = _params(_arr(a.nu_log, (M,)).astype(np.float64), _arr(a.theta_log, (M,)).astype(np.float64), M)
        h0 = None if not a.h0_r else (_arr(a.h0_r, (B, M)), _arr(a.h0_i, (B, M)))
        reset = None if not a.reset else _arr(a.reset, (B, T), np.uint8) != 0
        ar, ai, _, _ = O.transition(eta, delta, P)
        hr, hi = O._scan(ar, ai, u[..., :M], u[..., M:], h0, reset)
        _arr(a.y, (B, T, M))[:] = hr
        _arr(a.y_im, (B, T, M))[:] = hi
        _arr(a.last_r, (B, M))[:] = hr[:, -1]
        _arr(a.last_i, (B, M))[:] = hi[:, -1]
        ctl = _arr(a.controls, (B, T, 16))
        ctl[..., 0] = ctl[..., 1] = np.exp(eta)   # saved as the kernels save them: (E, E, delta, delta, ...)
        ctl[..., 2] = ctl[..., 3] = delta
        ctl[..., 4:] = 0.0
        if reset is not None:
            ctl[..., 8] = ctl[..., 9] = (~reset).astype(np.float32)  # keep
        else:
            ctl[..., 8] = ctl[..., 9] = 1.0
        return 0

    def sparc_mixer_backward(self, ref, stream):
        a = ref._obj
        self.calls.append(("backward", a.content_linear))
        assert a.content_linear == 2 and a.grad_projections and not a.y
        B, T, W = a.batch, a.length, a.width
        M = W // 2
        u = _arr(a.x, (B, T, W)).astype(np.float64)
        ctl = _arr(a.controls, (B, T, 16)).astype(np.float64)
        eta, delta = np.log(ctl[..., 0]), ctl[..., 2]
        reset = ctl[..., 8] == 0.0
        reset = reset if reset.any() else None
        dy = _arr(a.dy, (B, T, W)).astype(np.float64)
        P = _params(_arr(a.nu_log, (M,)).astype(np.float64), _arr(a.theta_log, (M,)).astype(np.float64), M)
        h0 = None if not a.h0_r else (_arr(a.h0_r, (B, M)), _arr(a.h0_i, (B, M)))
        gl = None if not a.grad_last_r else (_arr(a.grad_last_r, (B, M)), _arr(a.grad_last_i, (B, M)))
        ar, ai, _, _ = O.transition(eta, delta, P)
        hr, hi = O._scan(ar, ai, u[..., :M], u[..., M:], h0, reset)
        sc = O.scan_backward(eta, delta, P, hr, hi, dy[..., :M], dy[..., M:], h0, gl, reset)
        dx = _arr(a.dx, (B, T, W))
        dx[..., :M], dx[..., M:] = sc["lam_r"], sc["lam_i"]
        dp = _arr(a.grad_projections, (B, T, 2))
        dp[..., 0], dp[..., 1] = sc["delta"], sc["eta"]
        _arr(a.grad_nu_log, (M,))[:] = sc["nu_log"]
        _arr(a.grad_theta_log, (M,))[:] = sc["theta_log"]
        for name in ("grad_write_log_gain", "grad_energy_response", "grad_write_phase_response",
                     "grad_write_radial_response"):
            _arr(getattr(a, name), (M,))[:] = 0.0
        if a.grad_h0_r:
            _arr(a.grad_h0_r, (B, M))[:] = sc["h0_r"]
            _arr(a.grad_h0_i, (B, M))[:] = sc["h0_i"]
        return 0


@pytest.fixture
def fake(monkeypatch):
    """sparc_b200.scan over the fake library: CPU tensors are let through, since the fake
    computes on host memory."""
    from sparc_b200 import _lib, scan

    lib = FakeLib()
    monkeypatch.setattr(_lib, "lib", lambda: lib)
    monkeypatch.setattr(_lib, "require_cuda", lambda t, name: None)
    monkeypatch.setattr(_lib, "stream_handle", lambda dev: 0)

    class _WS:
        def get(self, dev, n, kind="mixer"):
            return torch.zeros(n, dtype=torch.uint8)

    monkeypatch.setattr(_lib, "WORKSPACES", _WS())
    scan.fake_lib = lib
    return scan


def _golden_inputs(d):
    return {k: torch.tensor(d[k], dtype=torch.float32).requires_grad_(True)
            for k in ("eta", "delta", "write_r", "write_i", "h0_r", "h0_i", "p_nu_log", "p_theta_log")}


def _golden_loss(d, out_r, out_i, last_r, last_i):
    return ((out_r.double() * torch.tensor(d["d_out_r"])).sum() + (out_i.double() * torch.tensor(d["d_out_i"])).sum()
            + (last_r.double() * torch.tensor(d["d_last_r"])).sum()
            + (last_i.double() * torch.tensor(d["d_last_i"])).sum())


GOLDEN_GRADS = (("eta", "grad_eta"), ("delta", "grad_delta"), ("write_r", "grad_write_r"), ("write_i", "grad_write_i"),
                ("h0_r", "grad_h0_r"), ("h0_i", "grad_h0_i"), ("p_nu_log", "grad_nu_log"),
                ("p_theta_log", "grad_theta_log"))


def test_tiled_serial_scan_matches_reference_golden(fake, golden):
    d = golden("tiled_h0_reset")
    t = _golden_inputs(d)
    out_r, out_i, last_r, last_i = fake.sparc_tiled_serial_scan(
        t["eta"], t["delta"], t["p_nu_log"], t["p_theta_log"], t["write_r"], t["write_i"],
        segment_pos=torch.tensor(d["segment_pos"]), initial_state=(t["h0_r"], t["h0_i"]))
    assert out_r.dtype == torch.float32 and out_r.is_contiguous() and out_i.is_contiguous() and last_r.shape == (2, 6)
    for got, ref in ((out_r, "out_r"), (out_i, "out_i"), (last_r, "last_r"), (last_i, "last_i")):
        assert O.rel_l2(got.detach().double().numpy(), d[ref]) < 1e-5, ref
    _golden_loss(d, out_r, out_i, last_r, last_i).backward()
    for k, ref in GOLDEN_GRADS:
        assert O.rel_l2(t[k].grad.double().numpy(), d[ref]) < 1e-4, k
    assert fake.fake_lib.calls == [("forward", 2), ("backward", 2)]


def test_scan_variants_agree(fake, golden):
    d = golden("tiled_h0_reset")
    eta, delta = torch.tensor(d["eta"]).float(), torch.tensor(d["delta"]).float()
    nl, tl = torch.tensor(d["p_nu_log"]).float(), torch.tensor(d["p_theta_log"]).float()
    br, bi = torch.tensor(d["write_r"]).float(), torch.tensor(d["write_i"]).float()
    ref_r, ref_i = fake.sparc_scan(eta, delta, nl, tl, br, bi)
    # the oracle's scan of the same controls and writes (no h0, no resets)
    ar, ai, _, _ = O.transition(d["eta"], d["delta"], _params(d["p_nu_log"], d["p_theta_log"], 6))
    hr, hi = O._scan(ar, ai, d["write_r"], d["write_i"])
    assert O.rel_l2(ref_r.double().numpy(), hr) < 1e-5 and O.rel_l2(ref_i.double().numpy(), hi) < 1e-5
    o_r, o_i, l_r, l_i = fake.sparc_scan_with_last(eta, delta, nl, tl, br, bi)
    assert torch.equal(o_r, ref_r) and torch.equal(l_r, ref_r[:, -1]) and torch.equal(l_i, ref_i[:, -1])
    c_r, c_i = fake.sparc_chunk_scan(eta[:, :32], delta[:, :32], nl, tl, br[:, :32], bi[:, :32], chunk_size=32)
    assert torch.allclose(c_r, ref_r[:, :32], rtol=1e-6, atol=1e-7)
    y = fake.sparc_chunk_scan(eta[:, :32], delta[:, :32], nl, tl, br[:, :32], bi[:, :32], chunk_size=16,
                              fused_output_relu=True)
    assert torch.allclose(y, torch.cat((ref_r[:, :32], ref_i[:, :32]), -1).relu(), rtol=1e-6, atol=1e-7)
    # the dispatch: a whole number of chunks goes to the chunked scan, a partial chunk, resets or
    # an initial state to the tiled serial scan; the results are the same scan
    dr, di = fake.sparc_training_scan_dispatch(eta[:, :32], delta[:, :32], nl, tl, br[:, :32], bi[:, :32])
    assert torch.allclose(dr, ref_r[:, :32], rtol=1e-6, atol=1e-7) and torch.allclose(di, ref_i[:, :32], rtol=1e-6, atol=1e-7)
    seg = torch.tensor(d["segment_pos"])
    tr, ti = fake.sparc_training_scan_dispatch(eta, delta, nl, tl, br, bi, segment_pos=seg)
    s_r, s_i, _, _ = fake.sparc_tiled_serial_scan(eta, delta, nl, tl, br, bi, segment_pos=seg)
    assert torch.equal(tr, s_r) and torch.equal(ti, s_i)


def test_fused_write(fake, golden):
    """raw_x times sqrt(1 - e^{-2 nu}) + 1e-8 as the writes, the gradient reaching raw_x."""
    d = golden("tiled_h0_reset")
    eta, delta = torch.tensor(d["eta"]).float()[:, :32], torch.tensor(d["delta"]).float()[:, :32]
    nl, tl = torch.tensor(d["p_nu_log"]).float(), torch.tensor(d["p_theta_log"]).float()
    raw = torch.tensor(d["x"]).float()[:, :32].requires_grad_(True)
    out_r, out_i = fake.sparc_chunk_scan(eta, delta, nl, tl, None, None, chunk_size=16, raw_x=raw, fused_write=True)
    gamma = torch.sqrt(1.0 - torch.exp(-2.0 * torch.exp(nl))) + 1e-8
    ref_r, ref_i = fake.sparc_scan(eta, delta, nl, tl, raw[..., :6].detach() * gamma, raw[..., 6:].detach() * gamma)
    assert torch.allclose(out_r, ref_r, rtol=1e-6, atol=1e-7) and torch.allclose(out_i, ref_i, rtol=1e-6, atol=1e-7)
    (out_r.sum() + out_i.sum()).backward()
    assert raw.grad is not None and raw.grad.shape == raw.shape and bool(raw.grad.abs().sum() > 0)


def test_controls_outside_the_controller_range_pass_through(fake):
    """eta and delta far outside the module controller's range (|eta| < ln16, |delta| < pi/2)
    reach the kernels unchanged and the result is the oracle's scan of exactly those controls,
    with their gradients (the reference's sparc_scan takes any controls)."""
    B, L, M = 1, 6, 3
    eta = torch.tensor([[LN16, -LN16, 5.0, 0.3, -9.0, 0.0]], requires_grad=True)
    delta = torch.tensor([[HALF_PI, 2.0, -HALF_PI, 0.1, 7.5, -30.0]], requires_grad=True)
    nl, tl = torch.full((M,), -1.0), torch.full((M,), 0.2)
    br, bi = torch.randn(B, L, M), torch.randn(B, L, M)
    out_r, out_i = fake.sparc_scan(eta, delta, nl, tl, br, bi)
    P = _params(nl.double().numpy(), tl.double().numpy(), M)
    ed, dd = eta.detach().double().numpy(), delta.detach().double().numpy()
    ar, ai, _, _ = O.transition(ed, dd, P)
    hr, hi = O._scan(ar, ai, br.double().numpy(), bi.double().numpy())
    assert O.rel_l2(out_r.detach().double().numpy(), hr) < 1e-6 and O.rel_l2(out_i.detach().double().numpy(), hi) < 1e-6
    (out_r.sum() + out_i.sum()).backward()
    sc = O.scan_backward(ed, dd, P, hr, hi, np.ones((B, L, M)), np.ones((B, L, M)))
    assert O.rel_l2(eta.grad.double().numpy(), sc["eta"]) < 1e-6
    assert O.rel_l2(delta.grad.double().numpy(), sc["delta"]) < 1e-6
    assert float(delta.grad[0, 5]) != 0.0  # no clamp: a gradient at delta = -30 too


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


def test_module_level_aliases(fake, golden):
    import sparc_b200

    d = golden("tiled_h0_reset")
    args = [torch.tensor(d[k]).float() for k in ("eta", "delta", "p_nu_log", "p_theta_log", "write_r", "write_i")]
    a, b = fake.sparc_scan_precomputed_decay(*args), fake.sparc_scan(*args)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    m = sparc_b200.SPARCMixer(8)
    with pytest.raises(ValueError, match="batch, length, 8"):
        sparc_b200.run_sequence(m, torch.randn(2, 3, 6))
    sparc_b200.prepare_decode(m)
    assert m._inference_fused
