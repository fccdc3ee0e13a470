"""Pin the float64 oracle against golden vectors made by running the reference itself
(tests/golden/make_golden.py): its Triton kernels under the CPU interpreter and its eager path.

Tolerances: the reference's "float64" eager run still computes the controller projection and
the write path in float32 (forward/control.py:131-163), and its Triton kernels run in float32,
so agreement is expected at the float32 level, not float64. A formula error shows up as O(1).
"""
import numpy as np
import pytest
import torch

from oracle import sparc_oracle as O

MIXER_CASES = ["mixer_b2_t64_w16", "mixer_b3_t37_w10", "mixer_b2_t96_w64_c32"]
GRAD_NAMES = [k for k in O.PARAM_NAMES if k != "energy_response"]


def _params(d):
    return O.Params.from_mapping({k: d["p_" + k] for k in O.PARAM_NAMES})


@pytest.mark.parametrize("name", MIXER_CASES)
@pytest.mark.parametrize("src,tol", [("eager64", 2e-6), ("triton", 1e-5)])
def test_mixer_forward_backward(golden, name, src, tol):
    d = golden(name)
    p = _params(d)
    y, last, _ = O.sparc_forward(d["x"], p)
    g = O.sparc_backward(d["x"], p, d["dy"])
    assert O.rel_l2(y, d[src + "_y"]) < tol
    assert O.rel_l2(g["x"], d[src + "_grad_x"]) < tol
    for k in GRAD_NAMES:
        assert O.rel_l2(g[k], d[src + "_grad_" + k]) < 3 * tol, k
    assert np.all(g["energy_response"] == 0)
    assert np.all(d[src + "_grad_energy_response"] == 0)


@pytest.mark.parametrize("name", MIXER_CASES)
def test_mixer_cache(golden, name):
    d = golden(name)
    _, last, _ = O.sparc_forward(d["x"], _params(d))
    assert O.rel_l2(last[0], d["triton_cache_last_r"]) < 1e-5
    assert O.rel_l2(last[1], d["triton_cache_last_i"]) < 1e-5


def test_mixer_bf16_inputs(golden):
    """bf16 activations: the oracle on the bf16 values matches the eager float64 run; the
    reference's own bf16 Triton path sits within a few percent (its own rounding error)."""
    d = golden("mixer_bf16_b2_t64_w32")
    p = _params(d)
    y, _, _ = O.sparc_forward(d["x"], p)
    g = O.sparc_backward(d["x"], p, d["dy"])
    assert O.rel_l2(y, d["eager64_y"]) < 2e-6
    assert O.rel_l2(g["x"], d["eager64_grad_x"]) < 2e-6
    assert O.rel_l2(y, d["triton_y"]) < 1e-2
    assert O.rel_l2(g["x"], d["triton_grad_x"]) < 6e-2


def test_decode(golden):
    d = golden("decode")
    p = _params(d)
    st = (d["state0_r"], d["state0_i"])
    ys = []
    for s in range(d["xs"].shape[0]):
        y, st = O.sparc_decode_step(d["xs"][s], p, st)
        ys.append(y)
    ys = np.stack(ys)
    for src in ("fused", "eager"):
        assert O.rel_l2(ys, d[src + "_ys"]) < 1e-5
        assert O.rel_l2(st[0], d[src + "_last_r"]) < 1e-5
        assert O.rel_l2(st[1], d[src + "_last_i"]) < 1e-5


def test_decode_equals_sequence(golden):
    """A chain of decode steps is the sequence scan of the stacked inputs."""
    d = golden("decode")
    p = _params(d)
    xs = d["xs"]
    st = (d["state0_r"], d["state0_i"])
    ys = []
    for s in range(xs.shape[0]):
        y, st = O.sparc_decode_step(xs[s], p, st)
        ys.append(y)
    yseq, last, _ = O.sparc_forward(np.transpose(xs, (1, 0, 2)), p, h0=(d["state0_r"], d["state0_i"]))
    np.testing.assert_allclose(np.transpose(np.stack(ys), (1, 0, 2)), yseq, rtol=0, atol=1e-12)
    np.testing.assert_allclose(st[0], last[0], atol=1e-12)


@pytest.mark.parametrize("src", ["chunk16", "serial"])
def test_real_scan(golden, src):
    d = golden("real")
    out, last = O.real_scan_forward(d["a"], d["b"])
    ga, gb = O.real_scan_backward(d["a"], d["b"], d["g"])
    assert O.rel_l2(out, d[src + "_out"]) < 1e-6
    assert O.rel_l2(ga, d[src + "_grad_a"]) < 1e-6
    assert O.rel_l2(gb, d[src + "_grad_b"]) < 1e-6
    assert O.rel_l2(last, d["with_last_last"]) < 1e-6


def test_real_scan_bf16(golden):
    d = golden("real")
    out, _ = O.real_scan_forward(d["bf16_a"], d["bf16_b"])
    ga, gb = O.real_scan_backward(d["bf16_a"], d["bf16_b"], d["g"])
    assert O.rel_l2(out, d["bf16_chunk16_out"]) < 1e-2
    assert O.rel_l2(ga, d["bf16_chunk16_grad_a"]) < 2e-2
    assert O.rel_l2(gb, d["bf16_chunk16_grad_b"]) < 1e-2


def test_h0_resets_and_grad_last(golden):
    """h0, segment resets and grad of the last state, against _SPARCTiledSerialScan
    (backward/scan.py:971-1070) run through the interpreter on the reference's own inputs."""
    d = golden("tiled_h0_reset")
    p = _params(d)
    # the oracle's scan on the reference's own controls/writes
    ar, ai, rho, z = O.transition(d["eta"], d["delta"], p)
    reset = d["segment_pos"] == 0
    hr, hi = O._scan(ar, ai, d["write_r"], d["write_i"], (d["h0_r"], d["h0_i"]), reset)
    assert O.rel_l2(hr, d["out_r"]) < 1e-5 and O.rel_l2(hi, d["out_i"]) < 1e-5
    assert O.rel_l2(hr[:, -1], d["last_r"]) < 1e-5
    # the scan adjoint with h0, resets and grad_last
    sc = O.scan_backward(d["eta"], d["delta"], p, hr, hi, d["d_out_r"], d["d_out_i"],
                         h0=(d["h0_r"], d["h0_i"]), grad_last=(d["d_last_r"], d["d_last_i"]),
                         reset=reset)
    for mine, ref in (("lam_r", "grad_write_r"), ("lam_i", "grad_write_i"), ("eta", "grad_eta"),
                      ("delta", "grad_delta"), ("nu_log", "grad_nu_log"),
                      ("theta_log", "grad_theta_log"), ("h0_r", "grad_h0_r"), ("h0_i", "grad_h0_i")):
        assert O.rel_l2(sc[mine], d[ref]) < 1e-5, mine
    # the module-level forward with h0 and resets reproduces the reference states
    _, last, S = O.sparc_forward(d["x"], p, h0=(d["h0_r"], d["h0_i"]), reset=reset)
    assert O.rel_l2(S["hr"], d["out_r"]) < 1e-5 and O.rel_l2(S["hi"], d["out_i"]) < 1e-5


def test_init_matches_reference(golden):
    import torch

    d = golden("init")
    for W in (16, 64):
        torch.manual_seed(0)
        p = O.init_params(W, lambda n: torch.rand(n).numpy())
        for k in O.PARAM_NAMES:
            np.testing.assert_allclose(p[k], d[f"w{W}_{k}"], rtol=1e-6, atol=1e-7)
    assert int(d["odd_raises"]) == 1
    with pytest.raises(ValueError):
        O.init_params(7, lambda n: np.zeros(n))


def _step_chain_grads(d, xs):
    """The oracle's adjoint of a chain of decode steps: the sequence scan over the steps with h0
    = the initial state and the gradient of the last state."""
    p = _params(d)
    x = np.transpose(xs, (1, 0, 2))  # [B, steps, W]
    dy = np.transpose(d["gs"], (1, 0, 2))
    h0 = (d["state0_r"], d["state0_i"])
    y, last, _ = O.sparc_forward(x, p, h0=h0)
    g = O.sparc_backward(x, p, dy, h0=h0, grad_last=(d["g_last_r"], d["g_last_i"]))
    return np.transpose(y, (1, 0, 2)), last, g


@pytest.mark.parametrize("src,tol", [("f64", 2e-6), ("f32", 1e-5)])
def test_eager_step_gradients(golden, src, tol):
    """The reference's differentiable eager step (forward/decode.py:296-306) chained over several
    steps: outputs, last state and the gradients of the inputs, the initial state and every
    parameter match the oracle's sequence adjoint with h0 and grad of the last state."""
    d = golden("decode_grad")
    ys, last, g = _step_chain_grads(d, d["xs"])
    assert O.rel_l2(ys, d[src + "_ys"]) < tol
    assert O.rel_l2(last[0], d[src + "_last_r"]) < tol and O.rel_l2(last[1], d[src + "_last_i"]) < tol
    assert O.rel_l2(np.transpose(g["x"], (1, 0, 2)), d[src + "_grad_xs"]) < tol
    assert O.rel_l2(g["h0_r"], d[src + "_grad_state0_r"]) < tol
    assert O.rel_l2(g["h0_i"], d[src + "_grad_state0_i"]) < tol
    for k in GRAD_NAMES:
        assert O.rel_l2(g[k], d[src + "_grad_" + k]) < 3 * tol, k


def test_eager_step_bf16_within_tolerance(golden):
    """With bfloat16 activations the reference rounds the write to bfloat16 (forward/control.py:163);
    its step then sits within the bf16 tolerance of the oracle on the same bf16 inputs."""
    d = golden("decode_grad")
    ys, last, g = _step_chain_grads(d, d["bf16_xs"])
    assert O.rel_l2(ys, d["bf16_ys"]) < 2e-2
    assert O.rel_l2(np.transpose(g["x"], (1, 0, 2)), d["bf16_grad_xs"]) < 2e-2
    for k in GRAD_NAMES:
        assert O.rel_l2(g[k], d["bf16_grad_" + k]) < 2e-2, k


@pytest.mark.parametrize("src", ["chunk16", "serial"])
def test_real_scan_mixed_dtypes(golden, src):
    """float32 retention with bfloat16 writes: the reference widens a from its own dtype, writes
    out (and grad_b) in b's dtype and grad_a in a's."""
    d = golden("real_mixed")
    out, last = O.real_scan_forward(d["a"], d["b"])
    ga, gb = O.real_scan_backward(d["a"], d["b"], d["g"])
    assert int(d[src + "_out_is_bf16"]) == 1 and int(d[src + "_grad_a_is_f32"]) == 1
    assert O.rel_l2(out, d[src + "_out"]) < 4e-3        # out rounded to bfloat16
    assert O.rel_l2(gb, d[src + "_grad_b"]) < 4e-3      # grad_b rounded to bfloat16
    # grad_a = lambda_t h_{t-1}: the reference takes h_{t-1} from its bfloat16 output
    assert O.rel_l2(ga, d[src + "_grad_a"]) < 1e-2
    assert O.rel_l2(last, d["with_last_last"]) < 1e-5  # last state in float32
    # rounding a to bfloat16 instead (what a same-dtype kernel would do) is far off
    a16 = d["a"].astype(np.float32).view(np.uint32)
    a16 = ((a16 + 0x7FFF + ((a16 >> 16) & 1)) & 0xFFFF0000).view(np.float32).astype(np.float64)
    out16, last16 = O.real_scan_forward(a16, d["b"])
    assert O.rel_l2(last16, d["with_last_last"]) > 1e-2


def test_complex_scan(golden):
    """The generic complex scan against the reference's float32 Triton kernels: forward, the
    last state and every gradient (the backward reading the forward's outputs as the previous
    states)."""
    d = golden("complex")
    out_r, out_i, last_r, last_i = O.complex_scan_forward(d["ar"], d["ai"], d["br"], d["bi"])
    assert O.rel_l2(out_r, d["f32_out_r"]) < 1e-5 and O.rel_l2(out_i, d["f32_out_i"]) < 1e-5
    assert O.rel_l2(last_r, d["with_last_last_r"]) < 1e-5 and O.rel_l2(last_i, d["with_last_last_i"]) < 1e-5
    assert np.array_equal(d["with_last_out_r"], d["f32_out_r"])
    grads = O.complex_scan_backward(d["ar"], d["ai"], d["f32_out_r"], d["f32_out_i"], d["gr"], d["gi"])
    for k, g in zip(("ar", "ai", "br", "bi"), grads):
        assert O.rel_l2(g, d["f32_grad_" + k]) < 1e-5, k


def test_complex_scan_bf16_writes(golden):
    """bfloat16 b with float32 a: out in bfloat16 (the reference's outputs are b's dtype), the
    gradients computed against those bfloat16 outputs and returned in a's dtype (float32)."""
    d = golden("complex")
    assert int(d["bf16b_out_dtype_is_b"]) == 1
    out_r, out_i, _, _ = O.complex_scan_forward(d["ar"], d["ai"], d["bf16b_br"], d["bf16b_bi"])
    assert O.rel_l2(out_r, d["bf16b_out_r"]) < 4e-3 and O.rel_l2(out_i, d["bf16b_out_i"]) < 4e-3
    # the output gradients reach the scan in the outputs' dtype (bfloat16)
    g16 = [torch.from_numpy(d[k]).to(torch.bfloat16).double().numpy() for k in ("gr", "gi")]
    grads = O.complex_scan_backward(d["ar"], d["ai"], d["bf16b_out_r"], d["bf16b_out_i"], *g16)
    # grad_b is returned in a's dtype (float32) and cast to b's by autograd
    for k, g, tol in zip(("ar", "ai", "br", "bi"), grads, (1e-5, 1e-5, 4e-3, 4e-3)):
        assert O.rel_l2(g, d["bf16b_grad_" + k]) < tol, k
