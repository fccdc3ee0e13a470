"""Bounds checks without a sanitizer: every output buffer is a view into a larger allocation
filled with a canary pattern, and after the call the canary on both sides must be intact (odd
shapes: modes not a multiple of the CTA's 256, lengths not a multiple of the chunk, one token,
widths of 2). Each entry point is called through the C ABI with such views."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

PAD = 4096  # elements of canary on each side


def _guarded(shape, dtype, fill=0.0):
    n = 1
    for s in shape:
        n *= s
    buf = torch.full((n + 2 * PAD,), float("nan") if dtype.is_floating_point else 0, dtype=dtype, device="cuda")
    if dtype.is_floating_point:
        buf.fill_(-12345.0)
    else:
        buf.fill_(0x5A5A5A5A)
    view = buf[PAD:PAD + n].view(shape)
    view.fill_(fill)
    return buf, view


def _intact(buf, dtype):
    head, tail = buf[:PAD], buf[-PAD:]
    want = -12345.0 if dtype.is_floating_point else 0x5A5A5A5A
    return bool((head == want).all()) and bool((tail == want).all())


@pytest.mark.parametrize("B,T,W,dtype", [(3, 37, 10, torch.float32), (2, 1, 2, torch.float32),
                                         (1, 100, 600, torch.bfloat16), (2, 33, 514, torch.float32)])
def test_mixer_forward_backward_stay_in_bounds(B, T, W, dtype):
    import sparc_b200
    from sparc_b200 import _lib

    L = _lib.lib()
    M = W // 2
    dt = _lib.dtype_code(dtype)
    torch.manual_seed(0)
    m = sparc_b200.SPARCMixer(W).cuda()
    p = [getattr(m, n).detach().float().contiguous() for n in ("nu_log", "theta_log", "phase_direction",
                                                              "radial_direction", "write_log_gain",
                                                              "write_phase_response", "write_radial_response")]
    x = torch.randn(B, T, W, device="cuda").to(dtype)
    chunks = L.sparc_mixer_carry_chunks(T, dt)
    yb, y = _guarded((B, T, W), dtype)
    cb, carry = _guarded((B, chunks, M, 2), torch.float32)
    kb, controls = _guarded((B, T, L.sparc_mixer_controls_floats()), torch.float32)
    lrb, lr = _guarded((B, M), torch.float32)
    lib_, li = _guarded((B, M), torch.float32)
    ws = torch.zeros(L.sparc_mixer_workspace_bytes(B, T, W, dt), dtype=torch.uint8, device="cuda")
    a = _lib.MixerFwdArgs(x.data_ptr(), y.data_ptr(), *[t.data_ptr() for t in p], None, None, lr.data_ptr(),
                          li.data_ptr(), carry.data_ptr(), controls.data_ptr(), None, None, 0.0, None, None, 0,
                          workspace=ws.data_ptr(), workspace_bytes=ws.numel(), batch=B, length=T, width=W,
                          dtype=dt, max_spin=0)
    assert L.sparc_mixer_forward(ctypes.byref(a), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    for buf, d in ((yb, dtype), (cb, torch.float32), (kb, torch.float32), (lrb, torch.float32), (lib_, torch.float32)):
        assert _intact(buf, d)
    dy = torch.randn(B, T, W, device="cuda").to(dtype)
    dxb, dx = _guarded((B, T, W), dtype)
    gbufs = []
    grads = []
    for n in (M, M, W + 1, W + 1, M, M, M, M):
        gb, g = _guarded((n,), torch.float32)
        gbufs.append(gb)
        grads.append(g)
    ba = _lib.MixerBwdArgs(x.data_ptr(), y.data_ptr(), dy.data_ptr(), dx.data_ptr(), *[t.data_ptr() for t in p],
                           None, None, None, None, None, None, carry.data_ptr(), controls.data_ptr(), None, None,
                           None, *[g.data_ptr() for g in grads], None, 0,
                           workspace=ws.data_ptr(), workspace_bytes=ws.numel(), batch=B, length=T, width=W,
                           dtype=dt, max_spin=0)
    assert L.sparc_mixer_backward(ctypes.byref(ba), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert _intact(dxb, dtype)
    for gb in gbufs:
        assert _intact(gb, torch.float32)


@pytest.mark.parametrize("B,L,D,dtype", [(2, 37, 300, torch.float32), (1, 16, 6, torch.bfloat16),
                                         (3, 50, 1030, torch.bfloat16)])
def test_real_scan_stays_in_bounds(B, L, D, dtype):
    from sparc_b200 import _lib

    lib = _lib.lib()
    dt = _lib.dtype_code(dtype)
    a = (torch.rand(B, L, D, device="cuda") * 0.5 + 0.45).to(dtype)
    b = torch.randn(B, L, D, device="cuda").to(dtype)
    ob, out = _guarded((B, L, D), dtype)
    cb, carry = _guarded((B, lib.sparc_real_carry_chunks(L), D), torch.float32)
    lb, last = _guarded((B, D), torch.float32)
    ws = torch.zeros(lib.sparc_real_workspace_bytes(B, L, D, dt), dtype=torch.uint8, device="cuda")
    f = _lib.RealFwdArgs(a.data_ptr(), b.data_ptr(), out.data_ptr(), last.data_ptr(), carry.data_ptr(),
                         ws.data_ptr(), ws.numel(), B, L, D, dt, dt, 0, 0, -1)
    assert lib.sparc_real_scan_forward(ctypes.byref(f), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert _intact(ob, dtype) and _intact(cb, torch.float32) and _intact(lb, torch.float32)
    g = torch.randn(B, L, D, device="cuda").to(dtype)
    gab, ga = _guarded((B, L, D), dtype)
    gbb, gb = _guarded((B, L, D), dtype)
    r = _lib.RealBwdArgs(a.data_ptr(), b.data_ptr(), g.data_ptr(), carry.data_ptr(), ga.data_ptr(), gb.data_ptr(),
                         ws.data_ptr(), ws.numel(), B, L, D, dt, dt, 0)
    assert lib.sparc_real_scan_backward(ctypes.byref(r), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert _intact(gab, dtype) and _intact(gbb, dtype)


@pytest.mark.parametrize("rows,n,k", [(130, 70, 24), (1, 300, 8)])
def test_gemm_stays_in_bounds(rows, n, k):
    from sparc_b200 import gemm

    a = torch.randn(rows, k, device="cuda").bfloat16()
    b = torch.randn(n, k, device="cuda").bfloat16()
    for dtype in (torch.float32, torch.bfloat16):
        ob, out = _guarded((rows, n), dtype)
        gemm.proj_gemm(a, b, dtype, out=out)
        torch.cuda.synchronize()
        assert _intact(ob, dtype)
        ref = a.float() @ b.float().t()
        assert float((out.float() - ref).norm() / ref.norm()) < 1e-2


@pytest.mark.parametrize("rows,n,k", [(72, 200, 24000), (136, 72, 24)])
def test_gemm_split_and_fused_stay_in_bounds(rows, n, k):
    """The split-k path (few output tiles, long k: the partials in the workspace, the finish
    launch writing the output) and the fused epilogue's staged vectors at ragged tile edges."""
    from sparc_b200 import gemm

    at = torch.randn(k, rows, device="cuda").bfloat16()  # token-major operands
    bt = torch.randn(k, n, device="cuda").bfloat16()
    x = torch.randn(rows, n, device="cuda").bfloat16()
    skip, c0, c1 = (torch.randn(n, device="cuda") for _ in range(3))
    dp = torch.randn(rows, 2, device="cuda")
    ref = at.float().t() @ bt.float() + skip * x.float() + dp[:, :1] * c0 + dp[:, 1:] * c1
    for dtype in (torch.float32, torch.bfloat16):
        ob, out = _guarded((rows, n), dtype)
        gemm.proj_gemm(at, bt, dtype, x=x, skip=skip, dp=dp, c0=c0, c1=c1, out=out, a_mn=True, b_mn=True)
        torch.cuda.synchronize()
        assert _intact(ob, dtype)
        assert float((out.float() - ref).norm() / ref.norm()) < 1e-2
    assert gemm.gemm_status("cuda") == 0


@pytest.mark.parametrize("rows,w,dtype", [(37, 2048, torch.bfloat16), (5, 700, torch.float32),
                                          (300, 10, torch.bfloat16)])
def test_rowdot_colsum_stay_in_bounds(rows, w, dtype):
    from sparc_b200 import _lib

    lib = _lib.lib()
    x = torch.randn(rows, w, device="cuda").to(dtype)
    dy = torch.randn(rows, w, device="cuda").to(dtype)
    dp = torch.randn(rows, 2, device="cuda")
    c = torch.randn(w + 1, 2, device="cuda")
    pb, p = _guarded((rows, 2), torch.float32)
    a = _lib.ProjRowdotArgs(x.data_ptr(), c.data_ptr(), p.data_ptr(), rows, w, _lib.dtype_code(dtype))
    assert lib.sparc_proj_rowdot(ctypes.byref(a), torch.cuda.current_stream().cuda_stream) == 0
    db, d_ctl = _guarded((w + 1, 2), torch.float32)
    sb, d_skip = _guarded((w,), torch.float32)
    wb, ws = _guarded((lib.sparc_proj_colsum_workspace_bytes(rows, w) // 4,), torch.float32)
    a = _lib.ProjColsumArgs(x.data_ptr(), dp.data_ptr(), dy.data_ptr(), d_ctl.data_ptr(), d_skip.data_ptr(),
                            ws.data_ptr(), ws.numel() * 4, rows, w, _lib.dtype_code(dtype))
    assert lib.sparc_proj_colsum(ctypes.byref(a), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert _intact(pb, torch.float32) and _intact(db, torch.float32) and _intact(sb, torch.float32)
    assert _intact(wb, torch.float32)
    xd = x.double()
    assert float((p.double() - (xd @ c[:w].double() + c[w].double())).norm()) < 1e-3 * float(p.double().norm())


@pytest.mark.parametrize("B,L,M,dtype", [(2, 37, 300, torch.float32), (1, 1, 1, torch.float32),
                                         (3, 70, 130, torch.bfloat16)])
def test_complex_scan_stays_in_bounds(B, L, M, dtype):
    from sparc_b200 import _lib

    lib = _lib.lib()
    dt = _lib.dtype_code(dtype)
    ar, ai = (torch.rand(B, L, M, device="cuda") * 0.6).to(dtype), (torch.rand(B, L, M, device="cuda") * 0.3).to(dtype)
    br, bi = torch.randn(B, L, M, device="cuda").to(dtype), torch.randn(B, L, M, device="cuda").to(dtype)
    orb, o_r = _guarded((B, L, M), dtype)
    oib, o_i = _guarded((B, L, M), dtype)
    lrb, l_r = _guarded((B, M), torch.float32)
    lib_, l_i = _guarded((B, M), torch.float32)
    wsb, ws = _guarded((lib.sparc_complex_workspace_bytes(B, L, M) // 4 + 4,), torch.float32)
    f = _lib.ComplexFwdArgs(ar.data_ptr(), ai.data_ptr(), br.data_ptr(), bi.data_ptr(), o_r.data_ptr(), o_i.data_ptr(),
                            l_r.data_ptr(), l_i.data_ptr(), ws.data_ptr(), ws.numel() * 4, B, L, M, dt, dt)
    assert lib.sparc_complex_scan_forward(ctypes.byref(f), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    for buf, t in ((orb, dtype), (oib, dtype), (lrb, torch.float32), (lib_, torch.float32), (wsb, torch.float32)):
        assert _intact(buf, t)
    gr, gi = torch.randn(B, L, M, device="cuda").to(dtype), torch.randn(B, L, M, device="cuda").to(dtype)
    gbufs = [_guarded((B, L, M), dtype) for _ in range(4)]
    r = _lib.ComplexBwdArgs(ar.data_ptr(), ai.data_ptr(), o_r.data_ptr(), o_i.data_ptr(), gr.data_ptr(), gi.data_ptr(),
                            *(v.data_ptr() for _, v in gbufs), ws.data_ptr(), ws.numel() * 4, B, L, M, dt, dt)
    assert lib.sparc_complex_scan_backward(ctypes.byref(r), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert all(_intact(b, dtype) for b, _ in gbufs) and _intact(wsb, torch.float32)


def test_rtrl_stays_in_bounds():
    import sparc_b200
    from sparc_b200 import _lib

    lib = _lib.lib()
    B, W, M = 3, 7, 131
    torch.manual_seed(0)
    cell = sparc_b200.SPARCRTRLCell(W, M).cuda()
    x = torch.randn(B, W, device="cuda")
    u = x @ torch.cat((cell.content_real, cell.content_imag), 1).detach()
    ctl = torch.stack((cell.phase_controller, cell.retention_controller), 1).detach()
    pj = (x @ ctl[:W] + ctl[W]).contiguous()
    state = torch.zeros(B, M, 2, device="cuda")
    shapes = [(B, M, 2)] * 5 + [(B, W, M, 2)] * 2 + [(B, W + 1, M, 2)] * 2
    tr = [torch.zeros(s, device="cuda") for s in shapes]
    outs = [_guarded(s, torch.float32) for s in shapes]
    nsb, ns = _guarded((B, M, 2), torch.float32)
    svb, saved = _guarded((B, M, lib.sparc_rtrl_saved_floats()), torch.float32)
    prm = [getattr(cell, n).detach().contiguous() for n in ("decay_log", "frequency_log", "write_log_gain",
                                                           "write_phase_response", "write_retention_response")]
    a = _lib.RtrlStepArgs(x.data_ptr(), u.contiguous().data_ptr(), pj.data_ptr(), None, state.data_ptr(),
                          ns.data_ptr(), *[t.data_ptr() for t in prm],
                          (ctypes.c_void_p * 9)(*[t.data_ptr() for t in tr]),
                          (ctypes.c_void_p * 9)(*[o[1].data_ptr() for o in outs]), saved.data_ptr(), B, W, M, 0)
    assert lib.sparc_rtrl_step(ctypes.byref(a), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert _intact(nsb, torch.float32) and _intact(svb, torch.float32)
    for ob, _ in outs:
        assert _intact(ob, torch.float32)
