"""GPU parity of the single-step decode paths.

* The differentiable step that SPARCMixer.step takes before prepare_inference() (the reference's
  eager step, forward/decode.py:296-306): outputs, the carried state and the gradients of the
  inputs, the initial state and every parameter over a chain of steps, against the reference's
  own eager run (tests/golden/decode_grad.npz) and the oracle's sequence adjoint; and a chain of
  steps against the full-sequence forward/backward with h0 on the GPU.
* Config 4 at its full size: 1024 fused decode steps (after prepare_inference) at batch 256,
  width 2048 with bfloat16 inputs and float32 state, against the module's full-sequence scan of
  the same inputs and against the float64 oracle on a few rows.

Tolerances (relative l2): float32 forward 1e-4, backward 1e-3; bfloat16 activations 2e-2.
"""
import numpy as np
import pytest
import torch

from oracle import sparc_oracle as O

pytestmark = pytest.mark.gpu

GRADS = [k for k in O.PARAM_NAMES if k != "energy_response"]


def _module(params: dict, width: int):
    import sparc_b200

    m = sparc_b200.SPARCMixer(width).cuda()
    with torch.no_grad():
        for k in O.PARAM_NAMES:
            getattr(m, k).copy_(torch.as_tensor(np.asarray(params[k]), dtype=torch.float32))
    return m


def _step_chain(m, xs, s0, gs, gl):
    """Steps over xs [steps, B, W] from s0 with autograd; loss = sum y_s . g_s + last . g_last."""
    xs = xs.clone().requires_grad_(True)
    st0 = (s0[0].clone().requires_grad_(True), s0[1].clone().requires_grad_(True))
    cur = st0
    ys = []
    loss = 0.0
    for k in range(xs.shape[0]):
        y, cur = m.step(xs[k], cur, None)
        ys.append(y)
        loss = loss + (y.double() * gs[k].double()).sum()
    loss = loss + (cur[0].double() * gl[0].double()).sum() + (cur[1].double() * gl[1].double()).sum()
    loss.backward()
    out = {"ys": torch.stack(ys).detach().double().cpu().numpy(),
           "last_r": cur[0].detach().double().cpu().numpy(), "last_i": cur[1].detach().double().cpu().numpy(),
           "grad_xs": xs.grad.double().cpu().numpy(),
           "grad_state0_r": st0[0].grad.double().cpu().numpy(), "grad_state0_i": st0[1].grad.double().cpu().numpy()}
    for k in O.PARAM_NAMES:
        out["grad_" + k] = getattr(m, k).grad.double().cpu().numpy()
    return out


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_eager_step_matches_reference_golden(golden, dtype):
    d = golden("decode_grad")
    W = d["xs"].shape[-1]
    m = _module({k: d["p_" + k] for k in O.PARAM_NAMES}, W)
    assert not m._inference_fused
    tag = "f32" if dtype == torch.float32 else "bf16"
    dev = "cuda"
    xs = torch.tensor(d[tag + "_xs"], device=dev).to(dtype)
    s0 = (torch.tensor(d["state0_r"], dtype=torch.float32, device=dev),
          torch.tensor(d["state0_i"], dtype=torch.float32, device=dev))
    gs = torch.tensor(d["gs"], device=dev)
    gl = (torch.tensor(d["g_last_r"], device=dev), torch.tensor(d["g_last_i"], device=dev))
    got = _step_chain(m, xs, s0, gs, gl)
    fwd, bwd = (1e-4, 1e-3) if dtype == torch.float32 else (2e-2, 2e-2)
    # against the reference's float64 eager run on the same (rounded) inputs
    if dtype == torch.float32:
        ref = {k[len("f64_"):]: d[k] for k in d.files if k.startswith("f64_")}
    else:
        # the float64 truth for the bf16 inputs: the oracle's sequence adjoint with h0
        p = O.Params.from_mapping({k: d["p_" + k] for k in O.PARAM_NAMES})
        x = np.transpose(d["bf16_xs"], (1, 0, 2))
        y, last, _ = O.sparc_forward(x, p, h0=(d["state0_r"], d["state0_i"]))
        g = O.sparc_backward(x, p, np.transpose(d["gs"], (1, 0, 2)), h0=(d["state0_r"], d["state0_i"]),
                             grad_last=(d["g_last_r"], d["g_last_i"]))
        ref = {"ys": np.transpose(y, (1, 0, 2)), "last_r": last[0], "last_i": last[1],
               "grad_xs": np.transpose(g["x"], (1, 0, 2)), "grad_state0_r": g["h0_r"], "grad_state0_i": g["h0_i"]}
        ref.update({"grad_" + k: g[k] for k in O.PARAM_NAMES})
    assert O.rel_l2(got["ys"], ref["ys"]) < fwd
    assert O.rel_l2(got["last_r"], ref["last_r"]) < fwd and O.rel_l2(got["last_i"], ref["last_i"]) < fwd
    for k in ["grad_xs", "grad_state0_r", "grad_state0_i"] + ["grad_" + n for n in GRADS]:
        e = O.rel_l2(got[k], ref[k])
        assert e < bwd, (k, e)
    assert np.all(got["grad_energy_response"] == 0)
    # and within tolerance of the reference's own run at this dtype
    for k in ["ys", "grad_xs"] + ["grad_" + n for n in GRADS]:
        e = O.rel_l2(got[k], d[tag + "_" + k])
        assert e < (1e-3 if dtype == torch.float32 else 2e-2), (k, e)


def test_eager_step_chain_equals_sequence_adjoint():
    """A chain of differentiable steps is the sequence forward/backward with h0 (same gradients)."""
    gen = torch.Generator().manual_seed(5)
    B, W, steps = 4, 512, 12
    M = W // 2
    torch.manual_seed(5)
    p = O.init_params(W, lambda n: torch.rand(n).numpy())
    p["phase_direction"] = (torch.randn(W + 1, generator=gen) / W ** 0.5).numpy()
    p["radial_direction"] = (torch.randn(W + 1, generator=gen) / W ** 0.5).numpy()
    p["write_phase_response"] = (torch.randn(M, generator=gen) * 0.8).numpy()
    p["write_radial_response"] = (torch.randn(M, generator=gen) * 0.8).numpy()
    m1 = _module(p, W)
    m2 = _module(p, W)
    xs = torch.randn(steps, B, W, generator=gen).cuda()
    gs = torch.randn(steps, B, W, generator=gen).cuda()
    s0 = (torch.randn(B, M, generator=gen).cuda() * 0.5, torch.randn(B, M, generator=gen).cuda() * 0.5)
    gl = (torch.randn(B, M, generator=gen).cuda(), torch.randn(B, M, generator=gen).cuda())
    got = _step_chain(m1, xs, s0, gs, gl)
    x = xs.transpose(0, 1).contiguous().requires_grad_(True)
    h0 = (s0[0].clone().requires_grad_(True), s0[1].clone().requires_grad_(True))
    y, cache = m2(x, return_cache=True, state=h0)
    loss = (y.double() * gs.transpose(0, 1).double()).sum() + (cache[0].double() * gl[0].double()).sum() \
        + (cache[1].double() * gl[1].double()).sum()
    loss.backward()
    assert O.rel_l2(got["ys"], y.detach().transpose(0, 1).double().cpu().numpy()) < 1e-5
    assert O.rel_l2(got["grad_xs"], x.grad.transpose(0, 1).double().cpu().numpy()) < 1e-5
    assert O.rel_l2(got["grad_state0_r"], h0[0].grad.double().cpu().numpy()) < 1e-5
    for k in GRADS:
        assert O.rel_l2(got["grad_" + k], getattr(m2, k).grad.double().cpu().numpy()) < 1e-5, k


def test_step_after_prepare_inference_has_no_autograd():
    """After prepare_inference() the fused kernel runs (no graph), as the reference's."""
    W, B = 64, 3
    p = O.init_params(W, lambda n: np.random.default_rng(0).random(n))
    m = _module(p, W)
    x = torch.randn(B, W, device="cuda", requires_grad=True)
    st = (torch.zeros(B, W // 2, device="cuda"), torch.zeros(B, W // 2, device="cuda"))
    y0, _ = m.step(x, st, None)
    assert y0.requires_grad
    m.prepare_inference()
    y1, _ = m.step(x, st, None)
    assert not y1.requires_grad
    assert O.rel_l2(y1.detach().double().cpu().numpy(), y0.detach().double().cpu().numpy()) < 1e-5


def test_decode_trajectory_config4():
    """Config 4: 1024 fused decode steps at batch 256, width 2048, bfloat16 inputs and float32
    state, against the full-sequence scan of the stacked inputs on the GPU (outputs and the final
    state) and against the float64 oracle on rows 0 and 255."""
    B, W, steps = 256, 2048, 1024
    torch.manual_seed(0)
    import sparc_b200

    m = sparc_b200.SPARCMixer(W).cuda()
    gen = torch.Generator(device="cuda").manual_seed(1)
    with torch.no_grad():  # controls and write responses away from zero so every term is live
        m.phase_direction.copy_(torch.randn(W + 1, generator=gen, device="cuda") / W ** 0.5)
        m.radial_direction.copy_(torch.randn(W + 1, generator=gen, device="cuda") / W ** 0.5)
        m.write_phase_response.copy_(torch.randn(W // 2, generator=gen, device="cuda") * 0.5)
        m.write_radial_response.copy_(torch.randn(W // 2, generator=gen, device="cuda") * 0.5)
    xs = torch.randn(steps, B, W, generator=gen, device="cuda").to(torch.bfloat16)
    m.prepare_inference()
    st = (torch.zeros(B, W // 2, device="cuda"), torch.zeros(B, W // 2, device="cuda"))
    ys = torch.empty_like(xs)
    with torch.no_grad():
        for s in range(steps):
            ys[s], st = m.step(xs[s], st, None)
        yseq, cache = m(xs.transpose(0, 1).contiguous(), return_cache=True)
    traj = ys.transpose(0, 1)
    e = ((traj.double() - yseq.double()).norm() / yseq.double().norm()).item()
    assert e < 2e-2, e
    for a, b in ((st[0], cache[0]), (st[1], cache[1])):
        assert ((a.double() - b.double()).norm() / b.double().norm()).item() < 1e-4
    P = O.Params.from_mapping({k: getattr(m, k).detach().double().cpu().numpy() for k in O.PARAM_NAMES})
    rows = [0, B - 1]
    xo = xs[:, rows].transpose(0, 1).double().cpu().numpy()
    y_ref, last_ref, _ = O.sparc_forward(xo, P)
    assert O.rel_l2(traj[rows].double().cpu().numpy(), y_ref) < 2e-2
    assert O.rel_l2(st[0][rows].double().cpu().numpy(), last_ref[0]) < 1e-4
    assert O.rel_l2(st[1][rows].double().cpu().numpy(), last_ref[1]) < 1e-4
