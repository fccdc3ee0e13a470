"""Generate the golden vectors in this folder by running the reference implementation itself.

Run from the repository root, in a container where the reference is mounted:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /path/to/reference [case ...]

(no case names: every case).
It imports the reference package ``sparc-kernal`` read-only and runs:

* its Triton kernels (the chunked SPARC scan, the tiled serial scan with h0/resets, the fused
  decode kernel, the write kernel, the real scans and the generic complex scan) under the Triton
  CPU interpreter
  (``TRITON_INTERPRET=1``), in float32 / bfloat16 exactly as they would run on a GPU;
* its eager torch path (``framework_eager`` backend) after ``module.double()``. Note that the
  reference casts the controller projection and the write path to float32 even then
  (forward/control.py:131-163), so this run is "mostly float64".

The vectors are small. They pin the float64 oracle in ``oracle/sparc_oracle.py`` (see
``tests/test_oracle_golden.py``) and serve as fixtures for the GPU parity tests. Nothing at
test time reads the reference: only the ``.npz`` files written here.
"""
from __future__ import annotations

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"
os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
PARAMS = (
    "nu_log", "theta_log", "phase_direction", "radial_direction", "write_log_gain",
    "energy_response", "write_phase_response", "write_radial_response",
)


def _np(t):
    return t.detach().to(torch.float64).cpu().numpy()


def _randomize(module, gen, scale=0.4):
    """Give every controller/response parameter non-zero values so all paths are exercised."""
    with torch.no_grad():
        W = module.width
        for name in ("phase_direction", "radial_direction"):
            p = getattr(module, name)
            p.copy_(torch.randn(p.shape, generator=gen) * scale / (W ** 0.5) * 3.0)
        module.write_phase_response.copy_(torch.randn(module.modes, generator=gen) * 0.8)
        module.write_radial_response.copy_(torch.randn(module.modes, generator=gen) * 0.8)
        module.write_log_gain.add_(torch.randn(module.modes, generator=gen) * 0.1)


def _run_mixer(sparc, state, x, dy, backend, dtype_params=torch.float32, return_cache=False):
    m = sparc.SPARCMixer(state["phase_direction"].numel() - 1)
    m.load_state_dict(state)
    m = m.to(dtype_params)
    m.set_scan_backend(backend)
    x = x.clone().requires_grad_(True)
    y, cache = m(x, return_cache=return_cache)
    out = {"y": _np(y)}
    if cache is not None:
        out["last_r"], out["last_i"] = _np(cache[0]), _np(cache[1])
    if y.requires_grad:
        (y.to(torch.float64) * dy.to(torch.float64)).sum().backward()
        out["grad_x"] = _np(x.grad)
        for n in PARAMS:
            g = getattr(m, n).grad
            out["grad_" + n] = _np(g) if g is not None else np.zeros(getattr(m, n).shape)
    return out


def mixer_case(sparc, name, B, T, W, seed, x_dtype=torch.float32, chunk_backend="chunk16"):
    torch.manual_seed(seed)
    base = sparc.SPARCMixer(W)
    gen = torch.Generator().manual_seed(seed + 1000)
    _randomize(base, gen)
    state = {k: v.clone() for k, v in base.state_dict().items()}
    x = torch.randn(B, T, W, generator=gen).to(x_dtype)
    dy = torch.randn(B, T, W, generator=gen).to(x_dtype)
    rec = {"x": _np(x), "dy": _np(dy)}
    for n in PARAMS:
        rec["p_" + n] = _np(state[n])
    eager64 = _run_mixer(sparc, state, x.to(torch.float64), dy, "framework_eager",
                         dtype_params=torch.float64)
    for k, v in eager64.items():
        rec["eager64_" + k] = v
    tri = _run_mixer(sparc, state, x, dy, chunk_backend)
    for k, v in tri.items():
        rec["triton_" + k] = v
    # forward with the cache through the reference's prefill path (no grad there for M<=512)
    cache = _run_mixer(sparc, state, x, dy, chunk_backend, return_cache=True)
    rec["triton_cache_last_r"] = cache["last_r"]
    rec["triton_cache_last_i"] = cache["last_i"]
    rec["triton_cache_y"] = cache["y"]
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)
    return rec


def init_case(sparc):
    rec = {}
    for W in (16, 64):
        torch.manual_seed(0)
        m = sparc.SPARCMixer(W)
        for k, v in m.state_dict().items():
            rec[f"w{W}_{k}"] = _np(v)
    try:
        sparc.SPARCMixer(7)
        rec["odd_raises"] = np.array(0)
    except ValueError:
        rec["odd_raises"] = np.array(1)
    np.savez_compressed(os.path.join(HERE, "init.npz"), **rec)


def _interpreter_libdevice():
    """The Triton CPU interpreter patches ``tl``/``tl.math`` but not ``libdevice``, whose
    functions then return None. Give the two the decode kernel calls (tanh, expm1) numpy
    bodies evaluated in the operand's precision, so the reference kernel can run unchanged."""
    from triton.language.extra import libdevice
    from triton.runtime.interpreter import TensorHandle
    import triton.language as tl

    def wrap(fn):
        def op(arg0, _semantic=None):
            h = arg0.handle
            data = fn(h.data).astype(h.data.dtype)
            return tl.core.tensor(TensorHandle(data, h.dtype.scalar), arg0.type)
        return op

    libdevice.tanh = wrap(np.tanh)
    libdevice.expm1 = wrap(np.expm1)


def decode_case(sparc):
    from forward.decode import latest_sparc_decode

    _interpreter_libdevice()

    B, W, steps, seed = 3, 16, 8, 7
    torch.manual_seed(seed)
    m = sparc.SPARCMixer(W)
    gen = torch.Generator().manual_seed(seed + 1000)
    _randomize(m, gen)
    xs = torch.randn(steps, B, W, generator=gen)
    rec = {"xs": _np(xs)}
    for n in PARAMS:
        rec["p_" + n] = _np(getattr(m, n))
    state0 = (torch.randn(B, W // 2, generator=gen) * 0.5, torch.randn(B, W // 2, generator=gen) * 0.5)
    rec["state0_r"], rec["state0_i"] = _np(state0[0]), _np(state0[1])
    with torch.no_grad():
        # eager step (the default before prepare_inference), forward/decode.py:296-306
        st = state0
        ys = []
        for s in range(steps):
            y, st = m.step(xs[s], st, None)
            ys.append(_np(y))
        rec["eager_ys"] = np.stack(ys)
        rec["eager_last_r"], rec["eager_last_i"] = _np(st[0]), _np(st[1])
        # fused Triton decode kernel, forward/decode.py:11-75
        m.prepare_inference()
        st = state0
        ys = []
        for s in range(steps):
            y, st = latest_sparc_decode(m, xs[s], st)
            ys.append(_np(y))
        rec["fused_ys"] = np.stack(ys)
        rec["fused_last_r"], rec["fused_last_i"] = _np(st[0]), _np(st[1])
    np.savez_compressed(os.path.join(HERE, "decode.npz"), **rec)


def decode_grad_case(sparc):
    """The eager step before prepare_inference (forward/decode.py:296-306) is differentiable:
    several steps with a carried state, loss = sum_s y_s . g_s + last . g_last, gradients of the
    inputs, the initial state and every parameter; in float32, with bfloat16 activations (the
    write is rounded to bfloat16 there, forward/control.py:163), and after module.double()."""
    B, W, steps, seed = 3, 16, 5, 17
    torch.manual_seed(seed)
    base = sparc.SPARCMixer(W)
    gen = torch.Generator().manual_seed(seed + 1000)
    _randomize(base, gen)
    state = {k: v.clone() for k, v in base.state_dict().items()}
    M = W // 2
    xs = torch.randn(steps, B, W, generator=gen)
    gs = torch.randn(steps, B, W, generator=gen)
    s0 = (torch.randn(B, M, generator=gen) * 0.5, torch.randn(B, M, generator=gen) * 0.5)
    gl = (torch.randn(B, M, generator=gen), torch.randn(B, M, generator=gen))
    rec = {"xs": _np(xs), "gs": _np(gs), "state0_r": _np(s0[0]), "state0_i": _np(s0[1]),
           "g_last_r": _np(gl[0]), "g_last_i": _np(gl[1])}
    for n in PARAMS:
        rec["p_" + n] = _np(state[n])
    for tag, x_dtype, p_dtype in (("f32", torch.float32, torch.float32),
                                  ("bf16", torch.bfloat16, torch.float32),
                                  ("f64", torch.float64, torch.float64)):
        m = sparc.SPARCMixer(W)
        m.load_state_dict(state)
        m = m.to(p_dtype)
        x = xs.to(x_dtype).clone().requires_grad_(True)
        st = (s0[0].to(p_dtype).clone().requires_grad_(True), s0[1].to(p_dtype).clone().requires_grad_(True))
        cur = st
        loss = 0.0
        ys = []
        for k in range(steps):
            y, cur = m.step(x[k], cur, None)
            ys.append(y)
            loss = loss + (y.to(torch.float64) * gs[k].to(torch.float64)).sum()
        loss = loss + (cur[0].to(torch.float64) * gl[0].to(torch.float64)).sum() \
            + (cur[1].to(torch.float64) * gl[1].to(torch.float64)).sum()
        loss.backward()
        rec[tag + "_xs"] = _np(x.detach())
        rec[tag + "_ys"] = _np(torch.stack(ys))
        rec[tag + "_last_r"], rec[tag + "_last_i"] = _np(cur[0]), _np(cur[1])
        rec[tag + "_grad_xs"] = _np(x.grad)
        rec[tag + "_grad_state0_r"], rec[tag + "_grad_state0_i"] = _np(st[0].grad), _np(st[1].grad)
        for n in PARAMS:
            g = getattr(m, n).grad
            rec[tag + "_grad_" + n] = _np(g) if g is not None else np.zeros(getattr(m, n).shape)
    np.savez_compressed(os.path.join(HERE, "decode_grad.npz"), **rec)


def real_mixed_case(sparc):
    """The real scans with float32 retention a and bfloat16 writes b: the reference loads a in its
    own dtype and widens it (forward/scan.py:631), writes out in b's dtype and grad_a in a's
    (backward/scan.py:815, 880). a is close to 1 over a long sequence, where rounding a to
    bfloat16 would change the recurrence."""
    from backward.scan import real_chunk_scan, real_scan, real_scan_with_last

    B, L, D = 2, 512, 24
    gen = torch.Generator().manual_seed(23)
    a = 0.99 + 0.0099 * torch.rand(B, L, D, generator=gen)
    b = (0.5 * torch.randn(B, L, D, generator=gen)).to(torch.bfloat16)
    g = torch.randn(B, L, D, generator=gen).to(torch.bfloat16)
    rec = {"a": _np(a), "b": _np(b), "g": _np(g)}
    for name, fn in (("chunk16", lambda a_, b_: real_chunk_scan(a_, b_, 16)),
                     ("serial", real_scan)):
        aa = a.clone().requires_grad_(True)
        bb = b.clone().requires_grad_(True)
        out = fn(aa, bb)
        out.backward(g)
        rec[name + "_out"] = _np(out)
        rec[name + "_out_is_bf16"] = np.array(int(out.dtype == torch.bfloat16))
        rec[name + "_grad_a"] = _np(aa.grad)
        rec[name + "_grad_a_is_f32"] = np.array(int(aa.grad.dtype == torch.float32))
        rec[name + "_grad_b"] = _np(bb.grad)
    out, last = real_scan_with_last(a, b)
    rec["with_last_out"], rec["with_last_last"] = _np(out), _np(last)
    np.savez_compressed(os.path.join(HERE, "real_mixed.npz"), **rec)


def complex_case(sparc):
    """The generic complex scans (complex_scan forward and backward, complex_scan_with_last):
    float32 throughout, and bfloat16 b with float32 a (out in b's dtype, every gradient in a's,
    the backward reading the bfloat16 outputs as the previous states). |a| close to 1 with a
    rotation, a ragged length, and modes beyond one 128-mode block."""
    from backward.scan import complex_scan, complex_scan_with_last

    B, L, M = 2, 40, 136
    gen = torch.Generator().manual_seed(31)
    rad = 0.9 + 0.099 * torch.rand(B, L, M, generator=gen)
    ang = 0.3 * torch.randn(B, L, M, generator=gen)
    ar, ai = rad * torch.cos(ang), rad * torch.sin(ang)
    br, bi = 0.5 * torch.randn(B, L, M, generator=gen), 0.5 * torch.randn(B, L, M, generator=gen)
    gr, gi = torch.randn(B, L, M, generator=gen), torch.randn(B, L, M, generator=gen)
    rec = {"ar": _np(ar), "ai": _np(ai), "br": _np(br), "bi": _np(bi), "gr": _np(gr), "gi": _np(gi)}
    for name, dt in (("f32", torch.float32), ("bf16b", torch.bfloat16)):
        t = [ar.clone().requires_grad_(True), ai.clone().requires_grad_(True),
             br.to(dt).clone().requires_grad_(True), bi.to(dt).clone().requires_grad_(True)]
        out_r, out_i = complex_scan(*t)
        (out_r.float() * gr).sum().backward(retain_graph=True)
        (out_i.float() * gi).sum().backward()
        rec[name + "_out_r"], rec[name + "_out_i"] = _np(out_r), _np(out_i)
        rec[name + "_out_dtype_is_b"] = np.array(int(out_r.dtype == dt))
        for k, tt in zip(("ar", "ai", "br", "bi"), t):
            rec[name + "_grad_" + k] = _np(tt.grad)
        if name == "bf16b":
            rec["bf16b_br"], rec["bf16b_bi"] = _np(t[2].detach()), _np(t[3].detach())
    o_r, o_i, l_r, l_i = complex_scan_with_last(ar, ai, br, bi)
    rec["with_last_out_r"], rec["with_last_out_i"] = _np(o_r), _np(o_i)
    rec["with_last_last_r"], rec["with_last_last_i"] = _np(l_r), _np(l_i)
    # every value here is a float32 (or bfloat16) value: stored as float32, exactly
    np.savez_compressed(os.path.join(HERE, "complex.npz"),
                        **{k: (v.astype(np.float32) if v.dtype == np.float64 else v) for k, v in rec.items()})


def real_case(sparc):
    from backward.scan import real_chunk_scan, real_scan, real_scan_with_last

    B, L, D = 2, 64, 24
    gen = torch.Generator().manual_seed(11)
    pre = torch.logit(0.9 + 0.099 * torch.rand(B, L, D, generator=gen))
    a = torch.sigmoid(pre)
    b = 0.5 * torch.randn(B, L, D, generator=gen)
    g = torch.randn(B, L, D, generator=gen)
    rec = {"a": _np(a), "b": _np(b), "g": _np(g)}
    for name, fn in (("chunk16", lambda a_, b_: real_chunk_scan(a_, b_, 16)),
                     ("serial", real_scan)):
        aa = a.clone().requires_grad_(True)
        bb = b.clone().requires_grad_(True)
        out = fn(aa, bb)
        (out * g).sum().backward()
        rec[name + "_out"] = _np(out)
        rec[name + "_grad_a"] = _np(aa.grad)
        rec[name + "_grad_b"] = _np(bb.grad)
    out, last = real_scan_with_last(a, b)
    rec["with_last_out"], rec["with_last_last"] = _np(out), _np(last)
    # bf16 activations, fp32 carry
    ab, bb_ = a.to(torch.bfloat16), b.to(torch.bfloat16)
    aa = ab.clone().requires_grad_(True)
    bb = bb_.clone().requires_grad_(True)
    out = real_chunk_scan(aa, bb, 16)
    (out.float() * g).sum().backward()
    rec["bf16_a"], rec["bf16_b"] = _np(ab), _np(bb_)
    rec["bf16_chunk16_out"] = _np(out)
    rec["bf16_chunk16_grad_a"] = _np(aa.grad)
    rec["bf16_chunk16_grad_b"] = _np(bb.grad)
    np.savez_compressed(os.path.join(HERE, "real.npz"), **rec)


def tiled_case(sparc):
    """h0 + segment resets + grad of the last state through _SPARCTiledSerialScan."""
    from backward.scan import sparc_tiled_serial_scan
    from forward.control import make_scan_inputs

    B, T, W, seed = 2, 40, 12, 5
    torch.manual_seed(seed)
    m = sparc.SPARCMixer(W)
    gen = torch.Generator().manual_seed(seed + 1000)
    _randomize(m, gen)
    M = W // 2
    x = torch.randn(B, T, W, generator=gen)
    h0r = torch.randn(B, M, generator=gen) * 0.5
    h0i = torch.randn(B, M, generator=gen) * 0.5
    seg = torch.ones(B, T, dtype=torch.int32)
    seg[0, 13] = 0
    seg[1, 27] = 0
    seg[1, 28] = 0
    dr = torch.randn(B, T, M, generator=gen)
    di = torch.randn(B, T, M, generator=gen)
    dlr = torch.randn(B, M, generator=gen)
    dli = torch.randn(B, M, generator=gen)
    rec = {"x": _np(x), "h0_r": _np(h0r), "h0_i": _np(h0i), "segment_pos": seg.numpy().astype(np.int64),
           "d_out_r": _np(dr), "d_out_i": _np(di), "d_last_r": _np(dlr), "d_last_i": _np(dli)}
    for n in PARAMS:
        rec["p_" + n] = _np(getattr(m, n))
    eta, delta, wr, wi = make_scan_inputs(m, x)
    eta = eta.detach().clone().requires_grad_(True)
    delta = delta.detach().clone().requires_grad_(True)
    wr = wr.detach().clone().requires_grad_(True)
    wi = wi.detach().clone().requires_grad_(True)
    h0r_ = h0r.clone().requires_grad_(True)
    h0i_ = h0i.clone().requires_grad_(True)
    out_r, out_i, last_r, last_i = sparc_tiled_serial_scan(
        eta, delta, m.nu_log, m.theta_log, wr, wi, segment_pos=seg,
        initial_state=(h0r_, h0i_), block_size=32, reset_first=False)
    loss = (out_r * dr).sum() + (out_i * di).sum() + (last_r * dlr).sum() + (last_i * dli).sum()
    loss.backward()
    rec.update({"eta": _np(eta), "delta": _np(delta), "write_r": _np(wr), "write_i": _np(wi),
                "out_r": _np(out_r), "out_i": _np(out_i), "last_r": _np(last_r), "last_i": _np(last_i),
                "grad_eta": _np(eta.grad), "grad_delta": _np(delta.grad),
                "grad_write_r": _np(wr.grad), "grad_write_i": _np(wi.grad),
                "grad_h0_r": _np(h0r_.grad), "grad_h0_i": _np(h0i_.grad),
                "grad_nu_log": _np(m.nu_log.grad), "grad_theta_log": _np(m.theta_log.grad)})
    np.savez_compressed(os.path.join(HERE, "tiled_h0_reset.npz"), **rec)


CASES = {
    "init": init_case,
    "mixer": lambda sparc: (
        mixer_case(sparc, "mixer_b2_t64_w16", 2, 64, 16, seed=1),
        mixer_case(sparc, "mixer_b3_t37_w10", 3, 37, 10, seed=2),
        mixer_case(sparc, "mixer_b2_t96_w64_c32", 2, 96, 64, seed=3, chunk_backend="chunk32"),
        mixer_case(sparc, "mixer_bf16_b2_t64_w32", 2, 64, 32, seed=4, x_dtype=torch.bfloat16)),
    "decode": decode_case,
    "decode_grad": decode_grad_case,
    "real": real_case,
    "real_mixed": real_mixed_case,
    "complex": complex_case,
    "tiled": tiled_case,
}


def main(reference_root: str, cases=()):
    sys.path.insert(0, os.path.join(reference_root, "sparc-kernal"))
    import sparc  # the reference module

    torch.set_num_threads(min(8, os.cpu_count() or 1))
    for name in (cases or CASES):
        CASES[name](sparc)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <reference checkout root> [case ...]  (cases: " + ", ".join(CASES) + ")")
    main(sys.argv[1], tuple(sys.argv[2:]))
