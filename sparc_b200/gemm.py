"""Host side of the projection variant's tensor-core products (``sparc_proj_gemm``, the tcgen05
kernel in csrc/proj_gemm.cu): out = a b^T (+ skip * x) (+ dp c^T) for bfloat16 operands, with
either operand K-major or stored transposed (the weight gradients, which contract over the
tokens), and the layer backward's skinny column sums (``sparc_proj_colsum``)."""
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
              c0=None, c1=None, out=None, a_mn: bool = False, b_mn: bool = False) -> torch.Tensor:
    """out[m, n] = sum_k a[m, k] b[n, k] (+ skip[n] x[m, n]) (+ dp[m, 0] c0[n] + dp[m, 1] c1[n]).

    a [rows, k], b [n, k] bfloat16 (contiguous), or stored transposed with a_mn (a [k, rows]) /
    b_mn (b [k, n]); float32 accumulation; out bfloat16 or float32. Products with few output
    tiles and a long k are split along k into the per-stream "gemm" workspace (the library
    chooses; the partials are summed in a fixed order). No autograd: the callers compose the
    products of the forward and backward themselves."""
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise TypeError("proj_gemm takes bfloat16 operands")
    if a.dim() != 2 or b.dim() != 2:
        raise ValueError("proj_gemm expects two matrices")
    ka = a.shape[0] if a_mn else a.shape[1]
    kb = b.shape[0] if b_mn else b.shape[1]
    if ka != kb:
        raise ValueError("proj_gemm: the contraction lengths of a and b differ")
    _lib.require_cuda(a, "a")
    _lib.require_cuda(b, "b")
    a = a.contiguous()
    b = b.contiguous()
    rows = a.shape[1] if a_mn else a.shape[0]
    n = b.shape[1] if b_mn else b.shape[0]
    k = ka
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
    L = _lib.lib()
    nbytes = L.sparc_proj_gemm_workspace_bytes(rows, n, k)  # split-k partials (0: unsplit)
    ws = _lib.WORKSPACES.get(a.device, nbytes, kind="gemm") if nbytes else None
    args = _lib.ProjGemmArgs(a.data_ptr(), b.data_ptr(), out.data_ptr(), _lib.ptr(x), _lib.ptr(skip), _lib.ptr(dp),
                             _lib.ptr(c0), _lib.ptr(c1), st.data_ptr(), rows, n, k,
                             1 if out.dtype == torch.float32 else 0, 0, int(a_mn), int(b_mn),
                             _lib.ptr(ws), 0 if ws is None else ws.numel())
    rc = L.sparc_proj_gemm(ctypes.byref(args), _lib.stream_handle(a.device))
    if rc != _lib.OK:
        msg = L.sparc_proj_gemm_last_error()
        raise RuntimeError(f"sparc_proj_gemm failed ({_lib.ERR_NAMES.get(rc, rc)}): {msg.decode() if msg else ''}")
    return out


def proj_colsum(x: torch.Tensor, dp: torch.Tensor, dy=None):
    """(d_ctl [w + 1, 2], d_skip [w] or None) float32: d_ctl[j] = sum_r x[r, j] dp[r, :] for
    j < w, d_ctl[w] = sum_r dp[r, :], d_skip[j] = sum_r dy[r, j] x[r, j]; x, dy [rows, w] float32
    or bfloat16, dp [rows, 2] float32 (sparc_proj_colsum: one pass, fixed order)."""
    L = _lib.lib()
    _lib.require_cuda(x, "x")
    x = x.contiguous()
    rows, w = x.shape
    dp = dp.detach().float().contiguous()
    if dy is not None:
        dy = dy.to(x.dtype).contiguous()
    d_ctl = torch.empty((w + 1, 2), dtype=torch.float32, device=x.device)
    d_skip = torch.empty(w, dtype=torch.float32, device=x.device) if dy is not None else None
    ws = torch.empty(L.sparc_proj_colsum_workspace_bytes(rows, w), dtype=torch.uint8, device=x.device)
    args = _lib.ProjColsumArgs(x.data_ptr(), dp.data_ptr(), _lib.ptr(dy), d_ctl.data_ptr(), _lib.ptr(d_skip),
                               ws.data_ptr(), ws.numel(), rows, w, _lib.dtype_code(x.dtype))
    rc = L.sparc_proj_colsum(ctypes.byref(args), _lib.stream_handle(x.device))
    if rc != _lib.OK:
        msg = L.sparc_proj_gemm_last_error()
        raise RuntimeError(f"sparc_proj_colsum failed ({_lib.ERR_NAMES.get(rc, rc)}): {msg.decode() if msg else ''}")
    return d_ctl, d_skip


def proj_rowdot(x: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
    """p [rows, 2] float32 = x c[:w] + c[w] for x [rows, w] (float32 or bfloat16) and c [w + 1, 2]
    (sparc_proj_rowdot: one warp per row, fixed order)."""
    _lib.require_cuda(x, "x")
    x = x.contiguous()
    rows, w = x.shape
    c = c.detach().float().contiguous()
    p = torch.empty((rows, 2), dtype=torch.float32, device=x.device)
    args = _lib.ProjRowdotArgs(x.data_ptr(), c.data_ptr(), p.data_ptr(), rows, w, _lib.dtype_code(x.dtype))
    rc = _lib.lib().sparc_proj_rowdot(ctypes.byref(args), _lib.stream_handle(x.device))
    if rc != _lib.OK:
        msg = _lib.lib().sparc_proj_gemm_last_error()
        raise RuntimeError(f"sparc_proj_rowdot failed ({_lib.ERR_NAMES.get(rc, rc)}): {msg.decode() if msg else ''}")
    return p


def pad8(t: torch.Tensor, dim: int = -1) -> torch.Tensor:
    """t with dimension `dim` zero-padded to a multiple of 8 (whole 16-byte rows of bfloat16 for
    the tensor maps); t itself when it already is one."""
    n = t.shape[dim]
    if n % 8 == 0:
        return t
    shape = list(t.shape)
    shape[dim] = -(-n // 8) * 8
    out = torch.zeros(shape, dtype=t.dtype, device=t.device)
    out.narrow(dim, 0, n).copy_(t)
    return out


def split3(t: torch.Tensor, role: str, dim: int = 1) -> torch.Tensor:
    """A float32 operand as three bfloat16 terms along its contraction dimension `dim` for a
    float32-accurate product on the bf16 tensor cores: t = hi + lo (hi = bf16(t),
    lo = bf16(t - hi), together 16 significand bits); an A operand becomes [hi | hi | lo], a B
    operand [hi | lo | hi], so that one product over 3k sums a_hi b_hi + a_hi b_lo + a_lo b_hi
    (the dropped a_lo b_lo is 2^-16 relative). dim = 1 for K-major operands, 0 for M/N-major."""
    t = t.detach().float().contiguous()
    hi = t.to(torch.bfloat16)
    lo = (t - hi.float()).to(torch.bfloat16)
    parts = (hi, hi, lo) if role == "a" else (hi, lo, hi)
    return torch.cat(parts, dim=dim).contiguous()


def proj_gemm_f32(a: torch.Tensor, b: torch.Tensor, dp=None, c0=None, c1=None, b_split=None,
                  a_mn: bool = False, b_mn: bool = False) -> torch.Tensor:
    """float32 out[m, n] = sum_k a[m, k] b[n, k] (+ dp[m, 0] c0[n] + dp[m, 1] c1[n]) for float32
    operands (a_mn / b_mn: stored transposed, as proj_gemm), through the three-term bf16 split
    (split3) in one tensor-core product; relative error ~1e-5. `b_split` may pass a cached
    split3(b, "b")."""
    sa = split3(a, "a", 0 if a_mn else 1)
    sb = split3(b, "b", 0 if b_mn else 1) if b_split is None else b_split
    return proj_gemm(sa, sb, torch.float32, dp=dp, c0=c0, c1=c1, a_mn=a_mn, b_mn=b_mn)
