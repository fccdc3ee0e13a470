"""The projection-variant oracle (oracle/jax_layer_oracle.py): pinned to the torch reference's
golden vectors through the selection identity, and its adjoints and RTRL traces checked by
central finite differences in float64."""
import numpy as np
import pytest

from oracle import jax_layer_oracle as J
from oracle import sparc_oracle as O

MIXER_CASES = ["mixer_b2_t64_w16", "mixer_b3_t37_w10", "mixer_b2_t96_w64_c32"]
NAME_MAP = {"decay_log": "nu_log", "frequency_log": "theta_log", "write_log_gain": "write_log_gain",
            "write_phase_response": "write_phase_response",
            "write_retention_response": "write_radial_response",
            "phase_controller": "phase_direction", "retention_controller": "radial_direction"}


def _params(d):
    return O.Params.from_mapping({k: d["p_" + k] for k in O.PARAM_NAMES})


@pytest.mark.parametrize("name", MIXER_CASES)
def test_selection_layer_is_the_reference_mixer(golden, name):
    """With content selecting x's halves and the readout selecting [Re h, Im h], relu of the
    layer is the torch reference's SPARCMixer output; its adjoint (fed the relu-masked
    gradient) is the reference's backward."""
    d = golden(name)
    p = _params(d)
    Jp = J.selection_params(p)
    y, _, _ = J.layer_forward(d["x"], Jp)
    assert O.rel_l2(np.maximum(y, 0.0), d["eager64_y"]) < 2e-6
    g = J.layer_backward(d["x"], Jp, d["dy"] * (y > 0))
    assert O.rel_l2(g["x"], d["eager64_grad_x"]) < 2e-6
    for jname, tname in NAME_MAP.items():
        assert O.rel_l2(g[jname], d["eager64_grad_" + tname]) < 6e-6, jname


def _rand_layer(rng, W, M):
    p = J.init_layer(W, M, rng)
    p["phase_controller"] = 0.3 * rng.standard_normal(W + 1)
    p["retention_controller"] = 0.3 * rng.standard_normal(W + 1)
    p["write_phase_response"] = 0.5 * rng.standard_normal(M)
    p["write_retention_response"] = 0.5 * rng.standard_normal(M)
    return p


def _fd(fn, arr, idx, eps=1e-6):
    old = arr[idx]
    arr[idx] = old + eps
    fp = fn()
    arr[idx] = old - eps
    fm = fn()
    arr[idx] = old
    return (fp - fm) / (2 * eps)


@pytest.mark.parametrize("act", ["tanh", "linear"])
@pytest.mark.parametrize("state", [False, True])
def test_layer_backward_finite_differences(act, state):
    rng = np.random.default_rng(3)
    B, T, W, M = 2, 6, 5, 4
    p = _rand_layer(rng, W, M)
    x = rng.standard_normal((B, T, W))
    dy = rng.standard_normal((B, T, W))
    h0 = (rng.standard_normal((B, M)), rng.standard_normal((B, M))) if state else None
    reset = np.zeros((B, T), bool)
    if state:
        reset[1, 3] = True
    gl = (rng.standard_normal((B, M)), rng.standard_normal((B, M))) if state else None

    def loss():
        y, last, _ = J.layer_forward(x, p, h0, reset, act)
        v = (y * dy).sum()
        if gl is not None:
            v += (last[0] * gl[0]).sum() + (last[1] * gl[1]).sum()
        return v

    g = J.layer_backward(x, p, dy, h0, gl, reset, act)
    for name in J.LAYER_NAMES:
        arr = p[name]
        for idx in [tuple(rng.integers(0, s) for s in arr.shape) for _ in range(3)]:
            assert abs(_fd(loss, arr, idx) - g[name][idx]) < 1e-6 * (1 + abs(g[name][idx])), (name, idx)
    for idx in [(0, 0, 1), (1, 4, 3), (1, 5, 0)]:
        assert abs(_fd(loss, x, idx) - g["x"][idx]) < 1e-6 * (1 + abs(g["x"][idx]))
    if state:
        for k, h in (("h0_r", h0[0]), ("h0_i", h0[1])):
            for idx in [(0, 1), (1, 3)]:
                assert abs(_fd(loss, h, idx) - g[k][idx]) < 1e-6 * (1 + abs(g[k][idx]))


def _run_cell(p, x, reset, act):
    B, T, W = x.shape
    M = p["decay_log"].shape[0]
    state = np.zeros((B, M), np.complex128)
    tr = J.init_traces(B, W, M)
    for t in range(T):
        state, tr = J.rtrl_step(p, state, tr, x[:, t], reset[:, t], act)
    return state, tr


@pytest.mark.parametrize("act", ["tanh", "linear"])
def test_rtrl_traces_are_the_state_sensitivities(act):
    """After T steps every trace is d h_T / d parameter (per mode; for the controllers summed
    over the modes it is the gradient of sum(h_T)), resets included."""
    rng = np.random.default_rng(5)
    B, T, W, M = 2, 5, 4, 3
    p = J.init_cell(W, M, rng, r_min=0.5, r_max=0.95)
    p["phase_controller"] = 0.4 * rng.standard_normal(W + 1)
    p["retention_controller"] = 0.4 * rng.standard_normal(W + 1)
    p["write_phase_response"] = 0.5 * rng.standard_normal(M)
    p["write_retention_response"] = 0.5 * rng.standard_normal(M)
    x = rng.standard_normal((B, T, W))
    reset = np.zeros((B, T), bool)
    reset[0, 2] = True
    _, tr = _run_cell(p, x, reset, act)
    wr, wi = rng.standard_normal((B, M)), rng.standard_normal((B, M))

    def probe():  # a real functional of the final state: sum(wr Re h + wi Im h)
        s, _ = _run_cell(p, x, reset, act)
        return (wr * s.real + wi * s.imag).sum()

    def from_trace(name, idx):
        t = tr[name]
        if t.ndim == 2:  # modal: d h_m / d param_m
            m = idx[0]
            return (wr[:, m] * t[:, m].real + wi[:, m] * t[:, m].imag).sum()
        if name in J.CONTENT_NAMES:  # d h_m / d param[j, m]
            j, m = idx
            return (wr[:, m] * t[:, j, m].real + wi[:, m] * t[:, j, m].imag).sum()
        j = idx[0]  # controller entry j affects every mode
        return (wr * t[:, j].real + wi * t[:, j].imag).sum()

    for name in J.MODAL_NAMES + J.CONTENT_NAMES + J.CONTROLLER_NAMES:
        arr = p[name]
        for idx in [tuple(rng.integers(0, s) for s in arr.shape) for _ in range(3)]:
            ref = _fd(probe, arr, idx)
            assert abs(ref - from_trace(name, idx)) < 1e-6 * (1 + abs(ref)), (name, idx)


def test_rtrl_grads():
    """Parameter gradients of a loss on the step's new state are Re(cot * trace) over the
    batch; the input gradient is the one-step pullback with the carry held fixed."""
    rng = np.random.default_rng(7)
    B, W, M = 3, 4, 5
    p = J.init_cell(W, M, rng, r_min=0.5, r_max=0.95)
    p["phase_controller"] = 0.4 * rng.standard_normal(W + 1)
    p["retention_controller"] = 0.4 * rng.standard_normal(W + 1)
    state = rng.standard_normal((B, M)) + 1j * rng.standard_normal((B, M))
    tr0 = {k: v + (rng.standard_normal(v.shape) + 1j * rng.standard_normal(v.shape)) * 0.1
           for k, v in J.init_traces(B, W, M).items()}
    x = rng.standard_normal((B, W))
    reset = np.array([False, True, False])
    gr, gi = rng.standard_normal((B, M)), rng.standard_normal((B, M))
    new_state, tr = J.rtrl_step(p, state, tr0, x, reset)
    g = J.rtrl_grads(p, state, tr, x, gr, gi, reset)
    for k, t in tr.items():
        if t.ndim == 2:
            ref = (gr * t.real + gi * t.imag).sum(0)
        elif k in J.CONTROLLER_NAMES:
            ref = (gr[:, None] * t.real + gi[:, None] * t.imag).sum((0, 2))
        else:
            ref = (gr[:, None] * t.real + gi[:, None] * t.imag).sum(0)
        assert np.allclose(g[k], ref, rtol=1e-12, atol=1e-12), k

    def step_loss():
        s, _ = J.rtrl_step(p, state, tr0, x, reset)
        return (gr * s.real + gi * s.imag).sum()

    for idx in [(0, 1), (1, 3), (2, 0)]:
        assert abs(_fd(step_loss, x, idx) - g["x"][idx]) < 1e-6 * (1 + abs(g["x"][idx]))
