"""CPU oracle for the SPARC hot path: a float64 numpy restatement of the reference.

TEST INFRASTRUCTURE ONLY. Nothing in the product path (the ``sparc_b200`` package and its
CUDA library) imports, calls or links this file. Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline / ``--impl reference`` legs use it, as the checker.

Parity pin: every function below is checked against golden vectors produced by running the
reference itself (its Triton kernels under the Triton CPU interpreter, and its eager torch
path); see ``tests/golden/make_golden.py`` and ``tests/test_oracle_golden.py``.

All citations are paths inside the reference project (Botwwt/sparc).

Math (one batch row, M = W/2 complex modes, t = 0..T-1):
    p0 = x_t . D0[:W] + D0[W],  p1 = x_t . D1[:W] + D1[W]        (D0 = phase, D1 = radial)
    eta = ln16 tanh(p1),  delta = (pi/2) tanh(p0)
    z = nu_m e^eta,  rho = e^-z,  phi = theta_m + (1 - rho) delta,  a = rho e^{i phi}
    gain = e^{wlg_m} sqrt(-expm1(-2z) / -expm1(-2 nu_m)) 2 sigmoid(tanh(p0) wpr_m + tanh(p1) wrr_m)
    b = gain (tanh(x_t[m]) + i tanh(x_t[M+m]))
    h_t = a_t h_{t-1} + b_t ,  y_t = relu([Re h_t, Im h_t])
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

LN16 = math.log(16.0)
HALF_PI = math.pi / 2.0

PARAM_NAMES = (
    "nu_log",
    "theta_log",
    "phase_direction",
    "radial_direction",
    "write_log_gain",
    "energy_response",
    "write_phase_response",
    "write_radial_response",
)


def _f64(a):
    return np.asarray(a, dtype=np.float64)


def _sigmoid(q):
    return 0.5 * (1.0 + np.tanh(0.5 * q))


@dataclass
class Params:
    """SPARCMixer parameters (sparc-kernal/sparc.py:59-88), as float64 arrays."""

    nu_log: np.ndarray
    theta_log: np.ndarray
    phase_direction: np.ndarray
    radial_direction: np.ndarray
    write_log_gain: np.ndarray
    energy_response: np.ndarray
    write_phase_response: np.ndarray
    write_radial_response: np.ndarray

    @classmethod
    def from_mapping(cls, m) -> "Params":
        return cls(**{k: _f64(m[k]) for k in PARAM_NAMES})

    @property
    def modes(self) -> int:
        return self.nu_log.shape[0]


def controls(x, P: Params):
    """Shared controls, forward/control.py:129-139 (make_controls).

    Returns eta, delta and the two tanh values (needed by the backward)."""
    x = _f64(x)
    p0 = x @ P.phase_direction[:-1] + P.phase_direction[-1]
    p1 = x @ P.radial_direction[:-1] + P.radial_direction[-1]
    tau0, tau1 = np.tanh(p0), np.tanh(p1)
    return LN16 * tau1, HALF_PI * tau0, tau0, tau1


def write_terms(x, eta, delta, P: Params):
    """Write gain and content, forward/control.py:150-163 (CPU branch) and the CUDA kernel
    _latest_write_forward forward/control.py:167-195.

    Returns (b_r, b_i, aux) with aux holding what the backward needs."""
    x = _f64(x)
    M = P.modes
    nu = np.exp(P.nu_log)
    z = nu * np.exp(eta)[..., None]
    num = -np.expm1(-2.0 * z)
    den = -np.expm1(-2.0 * nu)
    ratio = np.sqrt(num / den)
    phase, radial = delta / HALF_PI, eta / LN16
    q = phase[..., None] * P.write_phase_response + radial[..., None] * P.write_radial_response
    gate = 2.0 * _sigmoid(q)
    gain = np.exp(P.write_log_gain) * ratio * gate
    cr, ci = np.tanh(x[..., :M]), np.tanh(x[..., M:])
    aux = dict(z=z, num=num, den=den, nu=nu, gate=gate, gain=gain, cr=cr, ci=ci,
               phase=phase, radial=radial)
    return gain * cr, gain * ci, aux


def transition(eta, delta, P: Params):
    """Per-token transition a = rho e^{i phi}, forward/scan.py:1572-1575 (eager) and the chunk
    kernels forward/scan.py:925-942."""
    nu = np.exp(P.nu_log)
    theta = np.exp(P.theta_log)
    z = nu * np.exp(eta)[..., None]
    rho = np.exp(-z)
    phi = theta + (1.0 - rho) * delta[..., None]
    return rho * np.cos(phi), rho * np.sin(phi), rho, z


def _scan(ar, ai, br, bi, h0=None, reset=None):
    """Serial complex diagonal scan along axis 1, forward/scan.py:1355-1375
    (_eager_complex_scan) with the h0 / reset semantics of _sparc_tiled_serial_forward
    forward/scan.py:807-854 (reset zeroes a_t)."""
    B, T, M = br.shape
    hr = np.zeros((B, M)) if h0 is None else _f64(h0[0]).copy()
    hi = np.zeros((B, M)) if h0 is None else _f64(h0[1]).copy()
    out_r = np.empty((B, T, M))
    out_i = np.empty((B, T, M))
    for t in range(T):
        a_r, a_i = ar[:, t], ai[:, t]
        if reset is not None:
            keep = (~reset[:, t])[:, None]
            a_r, a_i = a_r * keep, a_i * keep
        nr = a_r * hr - a_i * hi + br[:, t]
        ni = a_i * hr + a_r * hi + bi[:, t]
        hr, hi = nr, ni
        out_r[:, t], out_i[:, t] = hr, hi
    return out_r, out_i


def sparc_forward(x, P: Params, h0=None, reset=None):
    """SPARCMixer.forward (sparc.py:90-91 -> forward/scan.py:1398-1603).

    x: [B, T, W]. Returns y [B, T, W], (last_r, last_i) [B, M] and the saved intermediates."""
    x = _f64(x)
    M = P.modes
    eta, delta, tau0, tau1 = controls(x, P)
    br, bi, waux = write_terms(x, eta, delta, P)
    ar, ai, rho, z = transition(eta, delta, P)
    hr, hi = _scan(ar, ai, br, bi, h0, reset)
    y = np.maximum(np.concatenate((hr, hi), axis=-1), 0.0)
    saved = dict(eta=eta, delta=delta, tau0=tau0, tau1=tau1, ar=ar, ai=ai, rho=rho, z=z,
                 hr=hr, hi=hi, waux=waux)
    assert y.shape[-1] == 2 * M
    return y, (hr[:, -1].copy(), hi[:, -1].copy()), saved


def scan_backward(eta, delta, P: Params, hr, hi, g_r, g_i, h0=None, grad_last=None, reset=None):
    """Adjoint of the SPARC scan alone (controls and writes treated as leaves).

    Follows the chunk reverse replay backward/scan.py:495-644 (adjoint update, grad_a, the
    radial/phase gradients at 593-638) and the tiled serial backward backward/scan.py:228-314
    (grad_last seeds the adjoint, grad_h0 is the adjoint that leaves t=0, a reset zeroes a_t and
    the control gradients at that step).

    g_r, g_i: [B, T, M] gradients arriving at the states. Returns a dict with lam_r/lam_i (the
    gradient of the writes), eta, delta [B, T], nu_log, theta_log [M], and h0_r/h0_i."""
    B, T, M = hr.shape
    ar, ai, rho, z = transition(eta, delta, P)
    theta = np.exp(P.theta_log)
    lam_r = np.zeros((B, M)) if grad_last is None else _f64(grad_last[0]).copy()
    lam_i = np.zeros((B, M)) if grad_last is None else _f64(grad_last[1]).copy()
    Lr = np.empty((B, T, M))
    Li = np.empty((B, T, M))
    for t in range(T - 1, -1, -1):
        lam_r = lam_r + g_r[:, t]
        lam_i = lam_i + g_i[:, t]
        Lr[:, t], Li[:, t] = lam_r, lam_i
        a_r, a_i = ar[:, t], ai[:, t]
        if reset is not None:
            keep = (~reset[:, t])[:, None]
            a_r, a_i = a_r * keep, a_i * keep
        # contribution to lambda_{t-1}: conj(a_t) * lambda_t
        lam_r, lam_i = a_r * lam_r + a_i * lam_i, -a_i * lam_r + a_r * lam_i
    if h0 is None:
        prev_r0 = np.zeros((B, 1, M))
        prev_i0 = np.zeros((B, 1, M))
    else:
        prev_r0 = _f64(h0[0])[:, None]
        prev_i0 = _f64(h0[1])[:, None]
    prev_r = np.concatenate((prev_r0, hr[:, :-1]), axis=1)
    prev_i = np.concatenate((prev_i0, hi[:, :-1]), axis=1)
    # gradient of a_t (backward/scan.py:593-594)
    gar = Lr * prev_r + Li * prev_i
    gai = -Lr * prev_i + Li * prev_r
    log_radius = -z
    radial_g = log_radius * (gar * ar + gai * ai)
    phase_g = -gar * ai + gai * ar
    radial_g = radial_g + (-log_radius) * rho * delta[..., None] * phase_g
    delta_g = phase_g * (1.0 - rho)
    if reset is not None:
        mask = (~reset)[..., None]
        radial_g, delta_g, phase_g = radial_g * mask, delta_g * mask, phase_g * mask
    out = dict(lam_r=Lr, lam_i=Li, eta_m=radial_g, delta_m=delta_g,
               eta=radial_g.sum(-1), delta=delta_g.sum(-1),
               nu_log=radial_g.sum((0, 1)), theta_log=theta * phase_g.sum((0, 1)))
    if h0 is not None:
        out["h0_r"], out["h0_i"] = lam_r, lam_i
    return out


def sparc_backward(x, P: Params, dy, h0=None, grad_last=None, reset=None):
    """Hand-derived adjoint of sparc_forward.

    The scan part is scan_backward. The write part follows backward/control.py:11-89
    (_latest_write_backward) and the controller part is torch autograd of make_controls
    forward/control.py:129-139. energy_response gets a zero gradient (forward/control.py:135
    multiplies it by 0). dy is the gradient of y = relu([Re h, Im h]).

    Returns a dict with 'x', every parameter name, and 'h0_r'/'h0_i' when h0 is given."""
    x = _f64(x)
    dy = _f64(dy)
    B, T, W = x.shape
    M = P.modes
    _, _, S = sparc_forward(x, P, h0, reset)
    hr, hi, z = S["hr"], S["hi"], S["z"]
    eta, delta, tau0, tau1 = S["eta"], S["delta"], S["tau0"], S["tau1"]
    wa = S["waux"]
    g_r = dy[..., :M] * (hr > 0)
    g_i = dy[..., M:] * (hi > 0)
    sc = scan_backward(eta, delta, P, hr, hi, g_r, g_i, h0, grad_last, reset)
    Lr, Li = sc["lam_r"], sc["lam_i"]
    grads = {}
    if h0 is not None:
        grads["h0_r"], grads["h0_i"] = sc["h0_r"], sc["h0_i"]

    # write path (backward/control.py:41-89)
    gain, gate, cr, ci = wa["gain"], wa["gate"], wa["cr"], wa["ci"]
    num, den, nu = wa["num"], wa["den"], wa["nu"]
    gain_g = gain * (Lr * cr + Li * ci)
    gate_g = gain_g * (1.0 - 0.5 * gate)
    dyn = z * np.exp(-2.0 * z) / num
    static = nu * np.exp(-2.0 * nu) / den
    eta_w = gain_g * dyn + gate_g * P.write_radial_response / LN16
    delta_w = gate_g * P.write_phase_response / HALF_PI
    dx = np.empty_like(x)
    dx[..., :M] = Lr * gain * (1.0 - cr * cr)
    dx[..., M:] = Li * gain * (1.0 - ci * ci)

    g_eta = sc["eta"] + eta_w.sum(-1)
    g_delta = sc["delta"] + delta_w.sum(-1)
    grads["nu_log"] = sc["nu_log"] + (gain_g * (dyn - static)).sum((0, 1))
    grads["theta_log"] = sc["theta_log"]
    grads["write_log_gain"] = gain_g.sum((0, 1))
    grads["write_phase_response"] = (gate_g * wa["phase"][..., None]).sum((0, 1))
    grads["write_radial_response"] = (gate_g * wa["radial"][..., None]).sum((0, 1))
    grads["energy_response"] = np.zeros(M)

    # controller (autograd of forward/control.py:130-139)
    dp1 = g_eta * LN16 * (1.0 - tau1 * tau1)
    dp0 = g_delta * HALF_PI * (1.0 - tau0 * tau0)
    dx += dp0[..., None] * P.phase_direction[:-1] + dp1[..., None] * P.radial_direction[:-1]
    gpd = np.empty(W + 1)
    grd = np.empty(W + 1)
    gpd[:W] = np.einsum("btw,bt->w", x, dp0)
    gpd[W] = dp0.sum()
    grd[:W] = np.einsum("btw,bt->w", x, dp1)
    grd[W] = dp1.sum()
    grads["phase_direction"] = gpd
    grads["radial_direction"] = grd
    grads["x"] = dx
    return grads


def sparc_decode_step(x, P: Params, state):
    """One fused decode step, forward/decode.py:11-55 (_latest_sparc_decode) and the eager
    step forward/decode.py:296-306. x: [B, W]; state: ([B, M], [B, M]).

    Returns (y [B, W], (new_r, new_i))."""
    y, last, _ = sparc_forward(_f64(x)[:, None], P, h0=state)
    return y[:, 0], last


def real_scan_forward(a, b, h0=None):
    """Real diagonal scan h_t = a_t h_{t-1} + b_t along axis 1.

    Serial kernel forward/scan.py:622-635 (_real_forward); the chunked kernels
    forward/scan.py:638-698 compute the same recurrence. Returns (out, last)."""
    a, b = _f64(a), _f64(b)
    B, L, D = a.shape
    h = np.zeros((B, D)) if h0 is None else _f64(h0).copy()
    out = np.empty((B, L, D))
    for t in range(L):
        h = a[:, t] * h + b[:, t]
        out[:, t] = h
    return out, h.copy()


def real_scan_backward(a, b, g):
    """Adjoint of real_scan_forward, backward/scan.py:35-55 (_real_backward) and the chunked
    reverse kernels backward/scan.py:61-128: lambda_t = g_t + a_{t+1} lambda_{t+1},
    grad_a_t = lambda_t h_{t-1} (h_{-1} = 0), grad_b_t = lambda_t."""
    a, b, g = _f64(a), _f64(b), _f64(g)
    out, _ = real_scan_forward(a, b)
    B, L, D = a.shape
    lam = np.zeros((B, D))
    ga = np.empty((B, L, D))
    gb = np.empty((B, L, D))
    for t in range(L - 1, -1, -1):
        lam = lam + g[:, t]
        prev = out[:, t - 1] if t > 0 else np.zeros((B, D))
        ga[:, t] = lam * prev
        gb[:, t] = lam
        lam = lam * a[:, t]
    return ga, gb


def complex_scan_forward(ar, ai, br, bi):
    """Generic complex diagonal scan h_t = a_t h_{t-1} + b_t (h_{-1} = 0) along axis 1,
    forward/scan.py:701-722 (_complex_forward). Returns (out_r, out_i, last_r, last_i)."""
    hr, hi = _scan(_f64(ar), _f64(ai), _f64(br), _f64(bi))
    return hr, hi, hr[:, -1].copy(), hi[:, -1].copy()


def complex_scan_backward(ar, ai, out_r, out_i, g_r, g_i):
    """Adjoint of complex_scan_forward as backward/scan.py:131-160 (_complex_backward) computes
    it, from the forward's outputs as the previous states: adj += g_t; grad_ar = Re(adj)
    Re(h_{t-1}) + Im(adj) Im(h_{t-1}); grad_ai = Im(adj) Re(h_{t-1}) - Re(adj) Im(h_{t-1});
    grad_b = adj; then adj = conj(a_t) adj. Returns (grad_ar, grad_ai, grad_br, grad_bi)."""
    ar, ai, out_r, out_i, g_r, g_i = (_f64(t) for t in (ar, ai, out_r, out_i, g_r, g_i))
    B, L, M = ar.shape
    adj_r = np.zeros((B, M))
    adj_i = np.zeros((B, M))
    gar, gai, gbr, gbi = (np.empty((B, L, M)) for _ in range(4))
    for t in range(L - 1, -1, -1):
        adj_r = adj_r + g_r[:, t]
        adj_i = adj_i + g_i[:, t]
        pr = out_r[:, t - 1] if t > 0 else np.zeros((B, M))
        pi = out_i[:, t - 1] if t > 0 else np.zeros((B, M))
        gar[:, t] = adj_r * pr + adj_i * pi
        gai[:, t] = -adj_r * pi + adj_i * pr
        gbr[:, t] = adj_r
        gbi[:, t] = adj_i
        adj_r, adj_i = ar[:, t] * adj_r + ai[:, t] * adj_i, -ai[:, t] * adj_r + ar[:, t] * adj_i
    return gar, gai, gbr, gbi


def rms_norm(x, weight, eps=1e-6):
    """RMSNorm used by the 4-layer stack workload (no reference counterpart)."""
    x = _f64(x)
    r = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    return x * r * _f64(weight)


def block_forward(x, P: Params, norm_weight, eps=1e-6, h0=None, reset=None):
    """One config-5 stack block: out = x + SPARCMixer(RMSNorm(x)), RMSNorm(x) = x r w with
    r = (mean(x^2) + eps)^(-1/2) per token (the stack's norm; no reference counterpart, the
    reference ships the mixer only). Returns (out, (last_r, last_i))."""
    x = _f64(x)
    n = rms_norm(x, norm_weight, eps)
    y, last, _ = sparc_forward(n, P, h0, reset)
    return x + y, last


def block_backward(x, P: Params, norm_weight, d_out, eps=1e-6, h0=None, grad_last=None, reset=None):
    """Adjoint of block_forward: the mixer's adjoint (sparc_backward) at the normalised input,
    then RMSNorm's, plus the residual path. Returns the mixer's gradients with 'x' replaced by
    the block input's gradient and 'norm_weight' added."""
    x = _f64(x)
    d_out = _f64(d_out)
    w = _f64(norm_weight)
    W = x.shape[-1]
    r = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    n = x * r * w
    g = sparc_backward(n, P, d_out, h0, grad_last, reset)
    dn = g["x"]
    s = (x * w * dn).sum(-1, keepdims=True)
    g["x"] = d_out + r * w * dn - (r ** 3 / W) * x * s
    g["norm_weight"] = (dn * x * r).sum((0, 1))
    return g


def init_params(width: int, rand_fn):
    """SPARCMixer.__init__ parameter construction, sparc.py:59-88.

    rand_fn(n) must return n uniform [0,1) samples in the reference's RNG order: the first call
    draws radius^2, the second draws the phase fraction. Returns a dict of float64 arrays."""
    if width % 2:
        raise ValueError("SPARC rnn_width must be even")
    M = width // 2
    tiny = np.finfo(np.float32).tiny
    r2 = np.maximum(_f64(rand_fn(M)), tiny)
    nu = -0.5 * np.log(r2)
    theta = np.maximum(2.0 * math.pi * _f64(rand_fn(M)), tiny)
    return dict(
        nu_log=np.log(nu),
        theta_log=np.log(theta),
        phase_direction=np.zeros(width + 1),
        radial_direction=np.zeros(width + 1),
        write_log_gain=np.log(np.sqrt(1.0 - np.exp(-2.0 * nu)) + 1e-8),
        energy_response=np.full(M, 0.5493061443340548),
        write_phase_response=np.zeros(M),
        write_radial_response=np.zeros(M),
    )


def rel_l2(a, b) -> float:
    a, b = _f64(a), _f64(b)
    den = np.linalg.norm(b.ravel())
    num = np.linalg.norm((a - b).ravel())
    return float(num / den) if den > 0 else float(num)


def max_rel(a, b) -> float:
    """max |a-b| / max |b| (a scale-aware max error)."""
    a, b = _f64(a), _f64(b)
    s = np.abs(b).max()
    d = np.abs(a - b).max()
    return float(d / s) if s > 0 else float(d)
