"""Generic complex diagonal scans h_t = a_t h_{t-1} + b_t (h_{-1} = 0): drop-ins for the
reference's ``complex_scan`` and ``complex_scan_with_last`` (backward/scan.py:887-919,
1653-1656, 1838-1855), on the sm_100a kernels of csrc/complex_scan.cu (chunk maps, the cluster
carry scan, replay; the backward likewise in reverse).

As in the reference: the four [B, L, M] operands are read in their own dtypes and widened to
float32, out_r / out_i have br's / bi's dtype, the last state is float32, the backward uses the
forward's outputs as the previous states and returns all four gradients in ar's dtype (autograd
casts each to its input's dtype). The kernels read each pair (ar, ai) and (br, bi) in one dtype:
a pair of two dtypes is widened to float32 first (exact), and outputs are cast to their own
dtypes after the kernel.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


def _check(ar, ai, br, bi):
    """The reference's shape check (ValueError), then the device (no CPU path)."""
    shape = ar.shape
    if any(t.shape != shape for t in (ai, br, bi)) or ar.ndim != 3:
        raise ValueError("complex scan expects matching [B, L, M] tensors")
    for name, t in (("ar", ar), ("ai", ai), ("br", br), ("bi", bi)):
        _lib.require_cuda(t, name)


def _pair(x, y):
    """One kernel dtype for a pair read together: its own, or float32 when the two differ."""
    if x.dtype == y.dtype:
        return x.contiguous(), y.contiguous()
    return x.float().contiguous(), y.float().contiguous()


def _workspace(device, B, L, M):
    L_ = _lib.lib()
    nbytes = L_.sparc_complex_workspace_bytes(B, L, M)
    if nbytes == 0:
        _lib.check(-2, "sparc_complex_workspace_bytes")
    return _lib.WORKSPACES.get(device, nbytes, kind="complex")


def _forward(ar, ai, br, bi, want_last):
    L_ = _lib.lib()
    kar, kai = _pair(ar, ai)
    kbr, kbi = _pair(br, bi)
    B, T, M = kbr.shape
    dev = kbr.device
    out_r = torch.empty_like(kbr)
    out_i = torch.empty_like(kbi)
    last_r = torch.empty((B, M), dtype=torch.float32, device=dev) if want_last else None
    last_i = torch.empty((B, M), dtype=torch.float32, device=dev) if want_last else None
    ws = _workspace(dev, B, T, M)
    args = _lib.ComplexFwdArgs(kar.data_ptr(), kai.data_ptr(), kbr.data_ptr(), kbi.data_ptr(), out_r.data_ptr(),
                               out_i.data_ptr(), _lib.ptr(last_r), _lib.ptr(last_i), ws.data_ptr(), ws.numel(),
                               B, T, M, _lib.dtype_code(kar.dtype), _lib.dtype_code(kbr.dtype))
    _lib.check(L_.sparc_complex_scan_forward(ctypes.byref(args), _lib.stream_handle(dev)),
               "sparc_complex_scan_forward")
    return out_r.to(br.dtype), out_i.to(bi.dtype), last_r, last_i


class _ComplexScanFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ar, ai, br, bi):
        out_r, out_i, _, _ = _forward(ar, ai, br, bi, False)
        ctx.save_for_backward(ar, ai, out_r, out_i)
        ctx.set_materialize_grads(False)
        return out_r, out_i

    @staticmethod
    def backward(ctx, g_r, g_i):
        L_ = _lib.lib()
        ar, ai, out_r, out_i = ctx.saved_tensors
        kar, kai = _pair(ar, ai)
        yr, yi = _pair(out_r, out_i)  # the previous states, as the forward returned them
        B, T, M = kar.shape
        dev = kar.device
        g_r = torch.zeros_like(yr) if g_r is None else g_r.to(yr.dtype).contiguous()
        g_i = torch.zeros_like(yi) if g_i is None else g_i.to(yi.dtype).contiguous()
        grads = [torch.empty_like(kar) for _ in range(4)]
        ws = _workspace(dev, B, T, M)
        args = _lib.ComplexBwdArgs(kar.data_ptr(), kai.data_ptr(), yr.data_ptr(), yi.data_ptr(), g_r.data_ptr(),
                                   g_i.data_ptr(), *(g.data_ptr() for g in grads), ws.data_ptr(), ws.numel(),
                                   B, T, M, _lib.dtype_code(kar.dtype), _lib.dtype_code(yr.dtype))
        _lib.check(L_.sparc_complex_scan_backward(ctypes.byref(args), _lib.stream_handle(dev)),
                   "sparc_complex_scan_backward")
        return tuple(g.to(ar.dtype) for g in grads)


def complex_scan(ar: torch.Tensor, ai: torch.Tensor, br: torch.Tensor, bi: torch.Tensor):
    """Differentiable complex scan (backward/scan.py:887-919, 1653-1656): (out_r, out_i)."""
    _check(ar, ai, br, bi)
    return _ComplexScanFunction.apply(ar, ai, br, bi)


@torch.no_grad()
def complex_scan_with_last(ar: torch.Tensor, ai: torch.Tensor, br: torch.Tensor, bi: torch.Tensor):
    """(out_r, out_i, last_r, last_i), the last state float32 (backward/scan.py:1838-1855)."""
    _check(ar, ai, br, bi)
    return _forward(ar, ai, br, bi, True)
