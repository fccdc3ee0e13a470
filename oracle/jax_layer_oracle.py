"""CPU oracle for the projection variant of SPARC (the JAX package ``sparc-impl``): the sequence
layer with content and readout matrices, and the RTRL cell's online traces.

TEST INFRASTRUCTURE ONLY. Nothing in the product path (the ``sparc_b200`` package and its
CUDA library) imports, calls or links this file. Only ``tests/`` uses it, as the checker.

Parity pin: JAX is not installed here, so the reference's JAX code cannot run. The layer below
reduces to the torch mixer (``sparc_oracle.sparc_forward``) when the content matrices select
x's halves and the readout selects [Re h, Im h] (``selection_params``): that composition is
checked against the golden vectors of the torch reference (``tests/test_oracle_jax.py``), which
pins the recurrence, controls and write gain. The content/readout products are plain matrix
products; the adjoints and the RTRL traces are checked by central finite differences in float64.
The JAX initializers' draws (``jax.random.PRNGKey``) cannot be reproduced without JAX: only
their distributions are restated (``init_layer``).

All citations are paths inside the reference project (Botwwt/sparc).

Layer math (sparc-impl/sparc/recurrence.py:20-63, layers.py:88-126), x: [B, T, W], M modes:
    p0 = [x, 1] . phase_controller,  p1 = [x, 1] . retention_controller
    u_r = x @ content_real,  u_i = x @ content_imag             ([W, M] each)
    c = tanh(u) (or u for content_activation "linear")
    a, gain as in the torch mixer (same controls, transition and write gain)
    h_t = a_t h_{t-1} + gain_t (c_r + i c_i)                     (associative scan, bptt.py:23-35)
    y = Re(h @ (readout_real + i readout_imag)^T) + skip * x
      = h_r @ readout_real^T - h_i @ readout_imag^T + skip * x
"""
from __future__ import annotations

import math

import numpy as np

from oracle import sparc_oracle as O

LN16 = O.LN16
HALF_PI = O.HALF_PI

MODAL_NAMES = ("decay_log", "frequency_log", "write_log_gain", "write_phase_response",
               "write_retention_response")  # recurrence.py:5-11
CONTENT_NAMES = ("content_real", "content_imag")  # recurrence.py:13
CONTROLLER_NAMES = ("phase_controller", "retention_controller")  # recurrence.py:14
LAYER_NAMES = MODAL_NAMES + CONTENT_NAMES + CONTROLLER_NAMES + ("readout_real", "readout_imag", "skip")


def _f64(a):
    return np.asarray(a, dtype=np.float64)


def mixer_params(J) -> O.Params:
    """The torch mixer's parameter set seen by the shared recurrence math
    (decay_log -> nu_log, frequency_log -> theta_log, the controllers -> the directions,
    write_retention_response -> write_radial_response; the JAX layer has no energy response)."""
    M = J["decay_log"].shape[0]
    return O.Params(nu_log=_f64(J["decay_log"]), theta_log=_f64(J["frequency_log"]),
                    phase_direction=_f64(J["phase_controller"]),
                    radial_direction=_f64(J["retention_controller"]),
                    write_log_gain=_f64(J["write_log_gain"]), energy_response=np.zeros(M),
                    write_phase_response=_f64(J["write_phase_response"]),
                    write_radial_response=_f64(J["write_retention_response"]))


def init_layer(model_width, modes, rng, r_min=0.9, r_max=0.999, max_phase=6.28):
    """Parameter distributions of SPARCSequenceLayer (layers.py:17-58, 112-124;
    initialization.py:5-39), drawn from a numpy Generator (JAX's PRNG is not reproducible)."""
    W, M = model_width, modes
    u = rng.random(M)
    decay_log = np.log(-0.5 * np.log(u * (r_max ** 2 - r_min ** 2) + r_min ** 2))
    frequency_log = np.log(max_phase * rng.random(M))
    nu, theta = np.exp(decay_log), np.exp(frequency_log)
    mag2 = np.abs(np.exp(-nu + 1j * theta)) ** 2
    return {
        "decay_log": decay_log,
        "frequency_log": frequency_log,
        "content_real": rng.standard_normal((W, M)) / math.sqrt(2.0 * W),
        "content_imag": rng.standard_normal((W, M)) / math.sqrt(2.0 * W),
        "phase_controller": np.zeros(W + 1),
        "retention_controller": np.zeros(W + 1),
        "write_log_gain": np.log(np.sqrt(1.0 - mag2)),
        "write_phase_response": np.zeros(M),
        "write_retention_response": np.zeros(M),
        "readout_real": rng.standard_normal((W, M)) / math.sqrt(M),
        "readout_imag": rng.standard_normal((W, M)) / math.sqrt(M),
        "skip": rng.standard_normal(W),
    }


def selection_params(P: O.Params):
    """Layer parameters under which the JAX layer computes the torch mixer's pre-relu output
    [Re h, Im h] from the same x (W = 2M): content selects x's halves, readout selects the
    state's parts, skip is zero."""
    M = P.modes
    W = 2 * M
    eye = np.eye(M)
    cr = np.zeros((W, M))
    ci = np.zeros((W, M))
    cr[:M] = eye
    ci[M:] = eye
    rr = np.zeros((W, M))
    ri = np.zeros((W, M))
    rr[:M] = eye
    ri[M:] = -eye  # Re(h * (0 - i)) = Im h
    return {"decay_log": P.nu_log, "frequency_log": P.theta_log, "content_real": cr,
            "content_imag": ci, "phase_controller": P.phase_direction,
            "retention_controller": P.radial_direction, "write_log_gain": P.write_log_gain,
            "write_phase_response": P.write_phase_response,
            "write_retention_response": P.write_radial_response, "readout_real": rr,
            "readout_imag": ri, "skip": np.zeros(W)}


def _gain_terms(eta, delta, P: O.Params):
    """Write gain without the content (recurrence.py:32-53; the torch restatement is
    sparc_oracle.write_terms)."""
    nu = np.exp(P.nu_log)
    z = nu * np.exp(eta)[..., None]
    num = -np.expm1(-2.0 * z)
    den = -np.expm1(-2.0 * nu)
    phase, radial = delta / HALF_PI, eta / LN16
    q = phase[..., None] * P.write_phase_response + radial[..., None] * P.write_radial_response
    gate = 2.0 * O._sigmoid(q)
    gain = np.exp(P.write_log_gain) * np.sqrt(num / den) * gate
    return dict(z=z, num=num, den=den, nu=nu, gate=gate, gain=gain, phase=phase, radial=radial)


def _content(u, activation):
    if activation == "tanh":
        return np.tanh(u)
    if activation == "linear":
        return u
    raise ValueError(activation)


def layer_forward(x, J, h0=None, reset=None, content_activation="tanh"):
    """SPARCSequenceLayer.__call__ (layers.py:97-126). Returns y [B, T, W], (last_r, last_i)
    and the saved intermediates."""
    x = _f64(x)
    P = mixer_params(J)
    eta, delta, tau0, tau1 = O.controls(x, P)
    ur, ui = x @ _f64(J["content_real"]), x @ _f64(J["content_imag"])
    cr, ci = _content(ur, content_activation), _content(ui, content_activation)
    ga = _gain_terms(eta, delta, P)
    ar, ai, rho, z = O.transition(eta, delta, P)
    hr, hi = O._scan(ar, ai, ga["gain"] * cr, ga["gain"] * ci, h0, reset)
    y = hr @ _f64(J["readout_real"]).T - hi @ _f64(J["readout_imag"]).T + _f64(J["skip"]) * x
    saved = dict(eta=eta, delta=delta, tau0=tau0, tau1=tau1, z=z, hr=hr, hi=hi, cr=cr, ci=ci,
                 ga=ga, P=P)
    return y, (hr[:, -1].copy(), hi[:, -1].copy()), saved


def layer_backward(x, J, dy, h0=None, grad_last=None, reset=None, content_activation="tanh"):
    """Adjoint of layer_forward (what jax.grad of the layer computes): the readout and skip
    products, the scan adjoint (sparc_oracle.scan_backward), the write path
    (backward/control.py:41-89 of the torch package restates the same derivative), the content
    products and the controllers. Returns a dict with 'x' and every layer parameter name
    (plus 'h0_r'/'h0_i' when h0 is given)."""
    x = _f64(x)
    dy = _f64(dy)
    B, T, W = x.shape
    _, _, S = layer_forward(x, J, h0, reset, content_activation)
    P, ga = S["P"], S["ga"]
    hr, hi, cr, ci = S["hr"], S["hi"], S["cr"], S["ci"]
    Rr, Ri = _f64(J["readout_real"]), _f64(J["readout_imag"])
    grads = {}
    # y = h_r Rr^T - h_i Ri^T + skip x
    g_r = dy @ Rr
    g_i = -(dy @ Ri)
    grads["readout_real"] = np.einsum("btw,btm->wm", dy, hr)
    grads["readout_imag"] = -np.einsum("btw,btm->wm", dy, hi)
    grads["skip"] = (dy * x).sum((0, 1))
    dx = _f64(J["skip"]) * dy

    sc = O.scan_backward(S["eta"], S["delta"], P, hr, hi, g_r, g_i, h0, grad_last, reset)
    Lr, Li = sc["lam_r"], sc["lam_i"]
    if h0 is not None:
        grads["h0_r"], grads["h0_i"] = sc["h0_r"], sc["h0_i"]
    gain, gate, num, den, nu, z = ga["gain"], ga["gate"], ga["num"], ga["den"], ga["nu"], ga["z"]
    gain_g = gain * (Lr * cr + Li * ci)
    gate_g = gain_g * (1.0 - 0.5 * gate)
    dyn = z * np.exp(-2.0 * z) / num
    static = nu * np.exp(-2.0 * nu) / den
    eta_w = gain_g * dyn + gate_g * P.write_radial_response / LN16
    delta_w = gate_g * P.write_phase_response / HALF_PI
    slope_r = 1.0 - cr * cr if content_activation == "tanh" else 1.0
    slope_i = 1.0 - ci * ci if content_activation == "tanh" else 1.0
    du_r = Lr * gain * slope_r
    du_i = Li * gain * slope_i
    dx += du_r @ _f64(J["content_real"]).T + du_i @ _f64(J["content_imag"]).T
    grads["content_real"] = np.einsum("btw,btm->wm", x, du_r)
    grads["content_imag"] = np.einsum("btw,btm->wm", x, du_i)

    g_eta = sc["eta"] + eta_w.sum(-1)
    g_delta = sc["delta"] + delta_w.sum(-1)
    grads["decay_log"] = sc["nu_log"] + (gain_g * (dyn - static)).sum((0, 1))
    grads["frequency_log"] = sc["theta_log"]
    grads["write_log_gain"] = gain_g.sum((0, 1))
    grads["write_phase_response"] = (gate_g * ga["phase"][..., None]).sum((0, 1))
    grads["write_retention_response"] = (gate_g * ga["radial"][..., None]).sum((0, 1))

    tau0, tau1 = S["tau0"], S["tau1"]
    dp1 = g_eta * LN16 * (1.0 - tau1 * tau1)
    dp0 = g_delta * HALF_PI * (1.0 - tau0 * tau0)
    dx += dp0[..., None] * P.phase_direction[:-1] + dp1[..., None] * P.radial_direction[:-1]
    for name, dp in (("phase_controller", dp0), ("retention_controller", dp1)):
        gc = np.empty(W + 1)
        gc[:W] = np.einsum("btw,bt->w", x, dp)
        gc[W] = dp.sum()
        grads[name] = gc
    grads["x"] = dx
    return grads


# ------------------------------------------------------------------------------------ RTRL
def init_cell(input_size, modes, rng, r_min=0.0, r_max=1.0, max_phase=6.28):
    """Parameter distributions of SPARCRTRLCell (layers.py:61-85 with _parameters 17-58):
    the layer's recurrent parameters, no readout or skip."""
    J = init_layer(input_size, modes, rng, r_min, r_max, max_phase)
    for k in ("readout_real", "readout_imag", "skip"):
        J.pop(k)
    return J


def init_traces(batch, input_size, modes):
    """rtrl.py:25-41: modal traces [B, M], content [B, W, M], controllers [B, W+1, M],
    complex, zero."""
    tr = {k: np.zeros((batch, modes), np.complex128) for k in MODAL_NAMES}
    tr.update({k: np.zeros((batch, input_size, modes), np.complex128) for k in CONTENT_NAMES})
    tr.update({k: np.zeros((batch, input_size + 1, modes), np.complex128) for k in CONTROLLER_NAMES})
    return tr


def _step_terms(J, x, content_activation):
    """Per-step quantities of recurrence_terms (recurrence.py:28-63) for x [B, W]."""
    P = mixer_params(J)
    eta, delta, tau0, tau1 = O.controls(x, P)
    ga = _gain_terms(eta, delta, P)
    ar, ai, rho, z = O.transition(eta, delta, P)
    ur, ui = x @ _f64(J["content_real"]), x @ _f64(J["content_imag"])
    cr, ci = _content(ur, content_activation), _content(ui, content_activation)
    return dict(P=P, eta=eta, delta=delta, tau0=tau0, tau1=tau1, a=ar + 1j * ai, rho=rho, z=z,
                ga=ga, c=cr + 1j * ci, cr=cr, ci=ci)


def rtrl_step(J, state, traces, x, reset=None, content_activation="tanh"):
    """One step of _trace_step (rtrl.py:61-108): the carry is zeroed where reset is set
    (_reset_carry, 142-151), then every trace is advanced as trace' = a trace + direct, with
    direct the forward-mode derivative of this step's h' = a h + gain c with respect to the
    parameter (for the controllers: w.r.t. the bias entry, spread over the inputs by the
    augmented input). Written out by hand here:

      decay_log:     a z (i rho delta - 1) h + gain (dyn - static) c
      frequency_log: i a theta h
      write_log_gain: gain c
      write_phase_response / write_retention_response: gain (1 - gate/2) tau0|tau1 c
      content_real[j] / content_imag[j]: gain slope_r x_j  /  i gain slope_i x_j
      phase_controller[j]: x_aug_j [i a (1 - rho)(pi/2) s0 h + gain (1 - gate/2) wpr s0 c]
      retention_controller[j]: x_aug_j [a z ln16 s1 (i rho delta - 1) h
                                        + gain (dyn ln16 s1 + (1 - gate/2) wrr s1) c]
    with s0 = 1 - tau0^2, s1 = 1 - tau1^2, dyn = z e^{-2z} / num, static = nu e^{-2nu} / den.

    state: complex [B, M]; x: [B, W]; reset: bool [B] or None. Returns (next_state, traces)."""
    x = _f64(x)
    state = np.asarray(state, np.complex128).copy()
    traces = {k: np.asarray(v, np.complex128).copy() for k, v in traces.items()}
    if reset is not None:
        keep = ~np.asarray(reset, bool)
        state *= keep[:, None]
        for k in traces:
            traces[k] *= keep.reshape((-1,) + (1,) * (traces[k].ndim - 1))
    s = _step_terms(J, x, content_activation)
    P, ga, a, c, z, rho = s["P"], s["ga"], s["a"], s["c"], s["z"], s["rho"]
    gain, gate, nu, num, den = ga["gain"], ga["gate"], ga["nu"], ga["num"], ga["den"]
    delta = s["delta"][:, None]
    tau0, tau1 = s["tau0"][:, None], s["tau1"][:, None]
    dyn = z * np.exp(-2.0 * z) / num
    static = nu * np.exp(-2.0 * nu) / den
    gq = gain * (1.0 - 0.5 * gate)
    theta = np.exp(P.theta_log)
    h = state
    direct = {
        "decay_log": a * z * (1j * rho * delta - 1.0) * h + gain * (dyn - static) * c,
        "frequency_log": 1j * a * theta * h,
        "write_log_gain": gain * c,
        "write_phase_response": gq * tau0 * c,
        "write_retention_response": gq * tau1 * c,
    }
    new = {k: a * traces[k] + direct[k] for k in MODAL_NAMES}
    slope_r = 1.0 - s["cr"] ** 2 if content_activation == "tanh" else np.ones_like(s["cr"])
    slope_i = 1.0 - s["ci"] ** 2 if content_activation == "tanh" else np.ones_like(s["ci"])
    new["content_real"] = a[:, None] * traces["content_real"] + (gain * slope_r)[:, None] * x[:, :, None]
    new["content_imag"] = a[:, None] * traces["content_imag"] + (1j * gain * slope_i)[:, None] * x[:, :, None]
    s0, s1 = 1.0 - tau0 ** 2, 1.0 - tau1 ** 2
    d_phase = 1j * a * (1.0 - rho) * HALF_PI * s0 * h + gq * P.write_phase_response * s0 * c
    d_ret = a * z * LN16 * s1 * (1j * rho * delta - 1.0) * h + (gain * dyn * LN16 * s1 + gq * P.write_radial_response * s1) * c
    aug = np.concatenate((x, np.ones((x.shape[0], 1))), axis=1)
    new["phase_controller"] = a[:, None] * traces["phase_controller"] + aug[:, :, None] * d_phase[:, None]
    new["retention_controller"] = a[:, None] * traces["retention_controller"] + aug[:, :, None] * d_ret[:, None]
    next_state = a * h + gain * c
    return next_state, new


def rtrl_grads(J, state, traces, x, g_r, g_i, reset=None, content_activation="tanh"):
    """Backward of stored_rtrl_step (rtrl.py:127-148) for a real loss of the step's new state:
    g_r, g_i = dL/d Re h', dL/d Im h' [B, M] (JAX's cotangent is g_r - i g_i). Parameter
    gradients are Re(cot * trace) summed over the batch (and over the modes for the
    controllers), with `traces` the step's NEW traces; the input gradient is the one-step
    pullback of h' = a h + gain c w.r.t. x with the (reset) carry state held fixed. Returns a
    dict with every recurrent parameter name and 'x'."""
    g_r = _f64(g_r)
    g_i = _f64(g_i)
    grads = {}
    for k, tr in traces.items():
        tr = np.asarray(tr, np.complex128)
        if tr.ndim == 2:
            grads[k] = (g_r * tr.real + g_i * tr.imag).sum(0)
        else:
            v = (g_r[:, None] * tr.real + g_i[:, None] * tr.imag).sum(0)
            grads[k] = v.sum(-1) if k in CONTROLLER_NAMES else v
    x = _f64(x)
    h = np.asarray(state, np.complex128)
    if reset is not None:
        h = h * (~np.asarray(reset, bool))[:, None]
    # one-step pullback through the same math as layer_backward with T = 1 and h0 = h
    Jl = dict(J)
    W = x.shape[1]
    M = g_r.shape[1]
    Jl["readout_real"] = np.zeros((W, M))
    Jl["readout_imag"] = np.zeros((W, M))
    Jl["skip"] = np.zeros(W)
    gl = layer_backward(x[:, None], Jl, np.zeros((x.shape[0], 1, W)), h0=(h.real, h.imag),
                        grad_last=(g_r, g_i), content_activation=content_activation)
    grads["x"] = gl["x"][:, 0]
    return grads
