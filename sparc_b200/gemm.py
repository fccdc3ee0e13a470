"""Host side of the projection variant's tensor-core products (``sparc_proj_gemm``, the tcgen05
kernel in csrc/proj_gemm.cu): out = a b^T (+ skip * x) (+ dp c^T) for bfloat16 operands."""
from __future__ import annotations

import ctypes

import torch

from . import _lib

_STATUS = {}


def _status(device: torch.device) -> torch.Tensor:
    key = (device.type, device.index)
    t = _STATUS.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _STATUS[key] = t
    return t


def gemm_status(device) -> int:
    """Bits set by a tensor-core product whose bounded wait ran out (0 when all is well)."""
    t = _STATUS.get((torch.device(device).type, torch.device(device).index))
    return 0 if t is None else int(t.item())


def supported(*dims: int) -> bool:
    """True when every contraction length is a whole number of 16-byte rows of bfloat16."""
    return all(d % 8 == 0 for d in dims)


def proj_gemm(a: torch.Tensor, b: torch.Tensor, out_dtype=torch.bfloat16, x=None, skip=None, dp=None,
              c0=None, c1=None, out=None) -> torch.Tensor:
    """out[m, n] = sum_k a[m, k] b[n, k] (+ skip[n] x[m, n]) (+ dp[m, 0] c0[n] + dp[m, 1] c1[n]).

    a [rows, k], b [n, k] bfloat16 (contiguous); float32 accumulation; out bfloat16 or float32.
    No autograd: the callers compose the products of the forward and backward themselves."""
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise TypeError("proj_gemm takes bfloat16 operands")
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[1]:
        raise ValueError("proj_gemm expects a [rows, k] and b [n, k]")
    _lib.require_cuda(a, "a")
    _lib.require_cuda(b, "b")
    a = a.contiguous()
    b = b.contiguous()
    rows, k = a.shape
    n = b.shape[0]
    if out is None:
        out = torch.empty((rows, n), dtype=out_dtype, device=a.device)
    if x is not None:
        x = x.to(torch.bfloat16).contiguous()
        skip = skip.detach().float().contiguous()
    if dp is not None:
        dp = dp.detach().float().contiguous()
        c0 = c0.detach().float().contiguous()
        c1 = c1.detach().float().contiguous()
    st = _status(a.device)
    args = _lib.ProjGemmArgs(a.data_ptr(), b.data_ptr(), out.data_ptr(), _lib.ptr(x), _lib.ptr(skip), _lib.ptr(dp),
                             _lib.ptr(c0), _lib.ptr(c1), st.data_ptr(), rows, n, k,
                             1 if out.dtype == torch.float32 else 0, 0)
    rc = _lib.lib().sparc_proj_gemm(ctypes.byref(args), _lib.stream_handle(a.device))
    if rc != _lib.OK:
        msg = _lib.lib().sparc_proj_gemm_last_error()
        raise RuntimeError(f"sparc_proj_gemm failed ({_lib.ERR_NAMES.get(rc, rc)}): {msg.decode() if msg else ''}")
    return out


def split3(t: torch.Tensor, role: str) -> torch.Tensor:
    """A float32 operand as three bfloat16 terms along k for a float32-accurate product on the
    bf16 tensor cores: t = hi + lo (hi = bf16(t), lo = bf16(t - hi), together 16 significand
    bits); an A operand becomes [hi | hi | lo], a B operand [hi | lo | hi], so that one product
    over 3k sums a_hi b_hi + a_hi b_lo + a_lo b_hi (the dropped a_lo b_lo is 2^-16 relative)."""
    t = t.detach().float().contiguous()
    hi = t.to(torch.bfloat16)
    lo = (t - hi.float()).to(torch.bfloat16)
    parts = (hi, hi, lo) if role == "a" else (hi, lo, hi)
    return torch.cat(parts, dim=1).contiguous()


def proj_gemm_f32(a: torch.Tensor, b: torch.Tensor, dp=None, c0=None, c1=None, b_split=None) -> torch.Tensor:
    """float32 out[m, n] = sum_k a[m, k] b[n, k] (+ dp[m, 0] c0[n] + dp[m, 1] c1[n]) for float32
    operands, through the three-term bf16 split (split3) in one tensor-core product; relative
    error ~1e-5. `b_split` may pass a cached split3(b, "b")."""
    return proj_gemm(split3(a, "a"), split3(b, "b") if b_split is None else b_split, torch.float32,
                     dp=dp, c0=c0, c1=c1)
