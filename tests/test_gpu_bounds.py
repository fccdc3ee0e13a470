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
