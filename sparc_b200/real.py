"""Real diagonal scans h_t = a_t h_{t-1} + b_t: drop-ins for the reference's ``real_scan``,
``real_chunk_scan`` and ``real_scan_with_last`` (backward/scan.py:1643-1650, 1821-1834).

All three run the same sm_100a kernels (the result does not depend on the chunk size, up to
float32 rounding); ``chunk_size`` is validated like the reference's, plus 128. As in the
reference, ``a`` keeps its own dtype (read and widened to float32 in the kernel,
forward/scan.py:631), the output has b's dtype, grad_a has a's and grad_b has b's
(backward/scan.py:815, 880); the recurrence is carried in float32.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


def _check(a, b, what, chunk_size=None):
    """Shape checks first (ValueError, as the reference's), then the device (no CPU path)."""
    if a.shape != b.shape or a.ndim != 3:
        raise ValueError(f"{what} expects matching [B, L, D] tensors")
    if chunk_size is not None and (chunk_size not in (16, 32, 64, 128) or a.shape[1] % chunk_size):
        raise ValueError("chunk size must be 16, 32, 64 or 128 and divide length")
    _lib.require_cuda(a, "a")
    _lib.require_cuda(b, "b")


def _forward(a, b, want_last, max_spin=0, inject_tile=None):
    L = _lib.lib()
    a = a.contiguous()
    b = b.contiguous()
    B, T, D = b.shape
    dt = _lib.dtype_code(b.dtype)
    adt = _lib.dtype_code(a.dtype)
    out = torch.empty_like(b)
    carry = torch.empty((B, L.sparc_real_carry_chunks(T), D), dtype=torch.float32, device=b.device)
    last = torch.empty((B, D), dtype=torch.float32, device=b.device) if want_last else None
    nbytes = L.sparc_real_workspace_bytes(B, T, D, dt)
    if nbytes == 0:
        _lib.check(-2, "sparc_real_workspace_bytes")
    ws = _lib.WORKSPACES.get(b.device, nbytes, kind="real")
    args = _lib.RealFwdArgs(a.data_ptr(), b.data_ptr(), out.data_ptr(), _lib.ptr(last), carry.data_ptr(),
                            ws.data_ptr(), ws.numel(), B, T, D, dt, adt, max_spin,
                            1 if inject_tile is not None else 0, inject_tile if inject_tile is not None else 0)
    _lib.check(L.sparc_real_scan_forward(ctypes.byref(args), _lib.stream_handle(b.device)),
               "sparc_real_scan_forward")
    return a, b, out, carry, last


class _RealScanFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b):
        a_c, b_c, out, carry, _ = _forward(a, b, False)
        ctx.save_for_backward(a_c, b_c, carry)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        L = _lib.lib()
        a, b, carry = ctx.saved_tensors
        B, T, D = b.shape
        dt = _lib.dtype_code(b.dtype)
        g = grad_out.to(b.dtype).contiguous()
        ga = torch.empty_like(a)
        gb = torch.empty_like(b)
        ws = _lib.WORKSPACES.get(b.device, L.sparc_real_workspace_bytes(B, T, D, dt), kind="real")
        args = _lib.RealBwdArgs(a.data_ptr(), b.data_ptr(), g.data_ptr(), carry.data_ptr(),
                                ga.data_ptr(), gb.data_ptr(), ws.data_ptr(), ws.numel(), B, T, D, dt,
                                _lib.dtype_code(a.dtype), 0)
        _lib.check(L.sparc_real_scan_backward(ctypes.byref(args), _lib.stream_handle(b.device)),
                   "sparc_real_scan_backward")
        return ga, gb


def real_scan(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Differentiable real scan (backward/scan.py:793-822, 1643-1644)."""
    _check(a, b, "real scan")
    return _RealScanFunction.apply(a, b)


def real_chunk_scan(a: torch.Tensor, b: torch.Tensor, chunk_size: int = 16) -> torch.Tensor:
    """Differentiable chunked real scan (backward/scan.py:825-884, 1647-1650)."""
    _check(a, b, "real chunk scan", chunk_size)
    return _RealScanFunction.apply(a, b)


@torch.no_grad()
def real_scan_with_last(a: torch.Tensor, b: torch.Tensor):
    """(out, last) without autograd (backward/scan.py:1821-1834); last is float32 [B, D]."""
    _check(a, b, "real scan")
    _, _, out, _, last = _forward(a, b, True)
    return out, last
