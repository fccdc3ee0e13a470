"""Scan-level functional entry points of the reference module: the SPARC recurrence from
precomputed per-token controls (eta, delta) [B, L] and writes (br, bi) [B, L, M], as
``sparc_scan``, ``sparc_chunk_scan``, ``sparc_scan_with_last``, ``sparc_tiled_serial_scan``,
``sparc_training_scan_dispatch`` and ``sparc_scan_precomputed_decay``
(sparc-kernal/backward/scan.py:1658-1877, re-exported by sparc.py:17-29):

    rho = exp(-nu e^eta),  phi = theta + (1 - rho) delta,  h_t = rho e^{i phi} h_{t-1} + b_t
    (nu = e^{nu_log}, theta = e^{theta_log}; forward/scan.py:725-757).

They run the mixer kernels in their scan-level mode (``content_linear = 2`` of the C ABI): the
controls (delta, eta) and the writes are read as given, for any values (the phase offset is
range-reduced before its sine and cosine), with no write gain; the outputs are written as two
contiguous [B, L, M] tensors. The only copies are the writes and, in the backward, the output
gradients laid side by side as [b_r | b_i] [B, L, 2M] rows for the kernels' tile loads, and the
controls stacked as float32 pairs [B, L, 2]. The gradients of eta, delta, the writes, nu_log,
theta_log and the initial state come from the mixer's backward kernels.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


def _io_dtype(dtype: torch.dtype) -> torch.dtype:
    return dtype if dtype in (torch.float32, torch.bfloat16) else torch.float32


def _scan_forward(eta, delta, nu_log, theta_log, br, bi, h0, reset):
    """sparc_mixer_forward in the scan-level mode: (out_r, out_i) [B, L, M] (the writes' dtype),
    the last state (float32) and what the backward needs."""
    L = _lib.lib()
    B, T, M = br.shape
    W = 2 * M
    io = _io_dtype(br.dtype)
    dev = br.device
    dt = _lib.dtype_code(io)
    u = torch.cat((br.to(io), bi.to(io)), dim=-1).contiguous()  # writes as [b_r | b_i] rows
    p = torch.stack((delta.detach().float(), eta.detach().float()), dim=-1).contiguous()
    nl = nu_log.detach().float().contiguous()
    tl = theta_log.detach().float().contiguous()
    zeros = torch.zeros(M, dtype=torch.float32, device=dev)  # write gain parameters: not read
    h0 = None if h0 is None else (h0[0].detach().float().contiguous(), h0[1].detach().float().contiguous())
    out_r = torch.empty((B, T, M), dtype=io, device=dev)
    out_i = torch.empty((B, T, M), dtype=io, device=dev)
    chunks = L.sparc_mixer_carry_chunks(T, dt)
    carry = torch.empty((B, chunks, M, 2), dtype=torch.float32, device=dev)
    controls = torch.empty((B, T, L.sparc_mixer_controls_floats()), dtype=torch.float32, device=dev)
    last_r = torch.empty((B, M), dtype=torch.float32, device=dev)
    last_i = torch.empty((B, M), dtype=torch.float32, device=dev)
    nbytes = L.sparc_mixer_workspace_bytes(B, T, W, dt)
    if nbytes == 0:
        _lib.check(-2, "sparc_mixer_workspace_bytes")
    ws = _lib.WORKSPACES.get(dev, nbytes)
    a = _lib.MixerFwdArgs(
        u.data_ptr(), out_r.data_ptr(), nl.data_ptr(), tl.data_ptr(), None, None,
        zeros.data_ptr(), zeros.data_ptr(), zeros.data_ptr(),
        _lib.ptr(h0[0] if h0 else None), _lib.ptr(h0[1] if h0 else None),
        last_r.data_ptr(), last_i.data_ptr(), carry.data_ptr(), controls.data_ptr(), _lib.ptr(reset),
        None, 0.0, None, p.data_ptr(), 2,
        ws.data_ptr(), ws.numel(), B, T, W, dt, 0, out_i.data_ptr())
    _lib.check(L.sparc_mixer_forward(ctypes.byref(a), _lib.stream_handle(dev)),
               "sparc_mixer_forward (scan-level mode)")
    return out_r, out_i, last_r, last_i, (u, nl, tl, zeros, h0, carry, controls)


def _scan_backward(saved, g_r, g_i, g_last_r, g_last_i):
    """sparc_mixer_backward in the scan-level mode: (d eta, d delta [B, L] float32, d nu_log,
    d theta_log [M], d b_r, d b_i [B, L, M] (views of one [B, L, 2M] buffer), d h0 or None)."""
    L = _lib.lib()
    u, nl, tl, zeros, h0, carry, controls = saved
    B, T, W = u.shape
    M = W // 2
    dev = u.device
    dt = _lib.dtype_code(u.dtype)
    zr = None
    if g_r is None or g_i is None:
        zr = torch.zeros((B, T, M), dtype=u.dtype, device=dev)
    dh = torch.cat(((zr if g_r is None else g_r).to(u.dtype), (zr if g_i is None else g_i).to(u.dtype)), dim=-1)
    dh = dh.contiguous()
    gl = None
    if g_last_r is not None or g_last_i is not None:
        gl = (torch.zeros((B, M), device=dev) if g_last_r is None else g_last_r.float().contiguous(),
              torch.zeros((B, M), device=dev) if g_last_i is None else g_last_i.float().contiguous())
    du = torch.empty_like(u)
    dp = torch.empty((B, T, 2), dtype=torch.float32, device=dev)
    g = [torch.empty(M, dtype=torch.float32, device=dev) for _ in range(6)]
    gh0 = None
    if h0 is not None:
        gh0 = (torch.empty((B, M), dtype=torch.float32, device=dev),
               torch.empty((B, M), dtype=torch.float32, device=dev))
    ws = _lib.WORKSPACES.get(dev, L.sparc_mixer_workspace_bytes(B, T, W, dt))
    a = _lib.MixerBwdArgs(
        u.data_ptr(), None, dh.data_ptr(), du.data_ptr(),
        nl.data_ptr(), tl.data_ptr(), None, None, zeros.data_ptr(), zeros.data_ptr(), zeros.data_ptr(),
        _lib.ptr(h0[0] if h0 else None), _lib.ptr(h0[1] if h0 else None),
        _lib.ptr(gl[0] if gl else None), _lib.ptr(gl[1] if gl else None),
        _lib.ptr(gh0[0] if gh0 else None), _lib.ptr(gh0[1] if gh0 else None),
        carry.data_ptr(), controls.data_ptr(), None, None, None,
        g[0].data_ptr(), g[1].data_ptr(), None, None, g[2].data_ptr(), g[5].data_ptr(),
        g[3].data_ptr(), g[4].data_ptr(), dp.data_ptr(), 2,
        workspace=ws.data_ptr(), workspace_bytes=ws.numel(), batch=B, length=T, width=W, dtype=dt, max_spin=0)
    _lib.check(L.sparc_mixer_backward(ctypes.byref(a), _lib.stream_handle(dev)),
               "sparc_mixer_backward (scan-level mode)")
    return dp[..., 1], dp[..., 0], g[0], g[1], du[..., :M], du[..., M:], gh0


class _SparcScanFunction(torch.autograd.Function):
    """Autograd op of the scan-level entry points: (out_r, out_i, last_r, last_i) from
    (eta, delta, nu_log, theta_log, br, bi) and an optional initial state; every input gets its
    gradient, including the initial state, and the last state's gradient flows back."""

    @staticmethod
    def forward(ctx, eta, delta, nu_log, theta_log, br, bi, h0_r, h0_i, reset):
        h0 = None if h0_r is None else (h0_r, h0_i)
        out_r, out_i, last_r, last_i, saved = _scan_forward(eta, delta, nu_log, theta_log, br, bi, h0, reset)
        ctx.saved = saved
        ctx.dtypes = (eta.dtype, delta.dtype, nu_log.dtype, theta_log.dtype, br.dtype, bi.dtype)
        ctx.set_materialize_grads(False)
        if out_r.dtype != br.dtype:
            out_r, out_i = out_r.to(br.dtype), out_i.to(bi.dtype)
        return out_r, out_i, last_r, last_i

    @staticmethod
    def backward(ctx, g_r, g_i, g_last_r, g_last_i):
        ge, gd, gn, gt, gbr, gbi, gh0 = _scan_backward(ctx.saved, g_r, g_i, g_last_r, g_last_i)
        ctx.saved = None
        grads = [t.to(d) for t, d in zip((ge, gd, gn, gt, gbr, gbi), ctx.dtypes)]
        return (*grads, gh0[0] if gh0 else None, gh0[1] if gh0 else None, None)


def _run(eta, delta, nu_log, theta_log, br, bi, h0=None, reset=None):
    """((out_r, out_i) in br's dtype, (last_r, last_i) float32)."""
    _lib.require_cuda(br, "the writes")
    h0_r, h0_i = (None, None) if h0 is None else h0
    out_r, out_i, last_r, last_i = _SparcScanFunction.apply(eta, delta, nu_log, theta_log, br, bi, h0_r, h0_i, reset)
    return (out_r, out_i), (last_r, last_i)


def _check(eta, delta, nu_log, theta_log, br, bi):
    """The reference's shape checks (backward/scan.py:925-931, 977-986)."""
    if eta.shape != delta.shape or eta.ndim != 2:
        raise ValueError("SPARC controls must be matching [B, L] tensors")
    if br.shape != bi.shape or br.ndim != 3:
        raise ValueError("SPARC writes must be matching [B, L, M] tensors")
    B, L, M = br.shape
    if eta.shape != (B, L) or nu_log.shape != (M,) or theta_log.shape != (M,):
        raise ValueError("SPARC control, spectrum and write shapes disagree")


def _fused_write(raw_x, nu_log):
    """Writes of the reference's fused-write path from raw_x [B, L, 2M]: each half times
    sqrt(1 - e^{-2 nu}) + 1e-8, rounded to raw_x's dtype (backward/scan.py:1153-1157, 1793-1798)."""
    M = nu_log.numel()
    gamma = torch.sqrt(1.0 - torch.exp(-2.0 * torch.exp(nu_log.float()))) + 1.0e-8
    return (raw_x[..., :M].float() * gamma).to(raw_x.dtype), (raw_x[..., M:].float() * gamma).to(raw_x.dtype)


def sparc_scan(eta, delta, nu_log, theta_log, br, bi):
    """Differentiable scan: (out_r, out_i) [B, L, M] in br's dtype (backward/scan.py:922-968,
    1658-1661). Any number of modes up to 2048 (the reference's serial kernel stops at 512)."""
    _check(eta, delta, nu_log, theta_log, br, bi)
    return _run(eta, delta, nu_log, theta_log, br, bi)[0]


@torch.no_grad()
def sparc_scan_with_last(eta, delta, nu_log, theta_log, br, bi):
    """(out_r, out_i, last_r, last_i) without autograd; the last states float32
    (backward/scan.py:1857-1877)."""
    if eta.shape != delta.shape or br.shape != bi.shape:
        raise ValueError("SPARC control or write shapes disagree")
    _check(eta, delta, nu_log, theta_log, br, bi)
    (out_r, out_i), (last_r, last_i) = _run(eta, delta, nu_log, theta_log, br, bi)
    return out_r, out_i, last_r, last_i


def sparc_tiled_serial_scan(eta, delta, nu_log, theta_log, br, bi, *, segment_pos=None, initial_state=None,
                            block_size: int = 128, reset_first: bool = False):
    """Differentiable scan with an initial state, segment resets (the transition is zero where
    segment_pos == 0, or at the first token with reset_first) and the last state:
    (out_r, out_i, last_r, last_i), gradients of every input including initial_state and of
    last (backward/scan.py:971-1070, 1664-1687). block_size is validated as the reference does
    and does not change the result."""
    from .mixer import reset_mask

    _check(eta, delta, nu_log, theta_log, br, bi)
    if block_size not in (32, 64, 128, 256):
        raise ValueError("block_size must be 32, 64, 128 or 256")
    B, L, M = br.shape
    if segment_pos is not None and segment_pos.numel() != 0 and segment_pos.shape != (B, L):
        raise ValueError("segment_pos must have shape [B,L]")
    if segment_pos is not None and segment_pos.numel() == 0:
        segment_pos = None
    h0 = None
    if initial_state is not None and initial_state[0].numel() != 0:
        if initial_state[0].shape != (B, M) or initial_state[1].shape != (B, M):
            raise ValueError("initial SPARC states must have shape [B,M]")
        h0 = (initial_state[0], initial_state[1])
    reset = reset_mask(segment_pos, bool(reset_first), (B, L), br.device)
    (out_r, out_i), (last_r, last_i) = _run(eta, delta, nu_log, theta_log, br, bi, h0, reset)
    return out_r, out_i, last_r, last_i


def _check_chunk_options(length, chunk_size, mode_block_size, backward_chunk_group, two_stage_spectral,
                         fused_output_relu, prefix_group_size, hierarchical_prefix):
    """The reference's validation of the chunked path's options (backward/scan.py:1146-1175);
    the options select among its kernels and do not change the result."""
    if chunk_size not in (16, 32, 64) or length % chunk_size:
        raise ValueError("chunk size must be 16, 32 or 64 and divide length")
    if mode_block_size not in (32, 64, 128, 256):
        raise ValueError("mode block size must be 32, 64, 128 or 256")
    if backward_chunk_group not in (1, 2):
        raise ValueError("backward chunk group must be 1 or 2")
    if (length // chunk_size) % backward_chunk_group:
        raise ValueError("backward chunk group must divide the chunk count")
    if backward_chunk_group > 1 and two_stage_spectral:
        raise ValueError("grouped replay and two-stage spectral are exclusive")
    if backward_chunk_group > 1 and fused_output_relu:
        raise ValueError("grouped replay and fused output are exclusive")
    if abs(prefix_group_size) not in (0, 32, 64, 128):
        raise ValueError("prefix group size must be 0, 32, 64 or 128")
    if prefix_group_size and not hierarchical_prefix:
        raise ValueError("a grouped prefix requires hierarchical_prefix")


def _no_fused_controller_backward(controller_backward_cache):
    if controller_backward_cache is not None:
        raise NotImplementedError(
            "controller_backward_cache (the reference's fused controller backward) is not supported: "
            "pass eta and delta with their autograd history instead")


def sparc_chunk_scan(eta, delta, nu_log, theta_log, br, bi, chunk_size: int = 32, hierarchical_prefix: bool = False,
                     precompute_shared: bool = False, compressed_transition: bool = False,
                     atomic_shared: bool = False, two_stage_spectral: bool = False,
                     compact_control_cache: bool = False, precompute_spectral: bool = False,
                     mode_block_size: int = 128, raw_x=None, fused_write: bool = False,
                     backward_chunk_group: int = 1, fused_output_relu: bool = False, prefix_group_size: int = 0,
                     controller_backward_cache=None):
    """Differentiable chunked scan (backward/scan.py:1124-1372, 1703-1751): (out_r, out_i), or
    relu([Re h, Im h]) [B, L, 2M] with fused_output_relu. With fused_write the writes come from
    raw_x (gradient to raw_x). The chunk and kernel-selection options are validated as the
    reference does; the result does not depend on them."""
    _no_fused_controller_backward(controller_backward_cache)
    if fused_write and raw_x is None:
        raise ValueError("raw_x is required by the fused-write SPARC path")
    if eta.shape != delta.shape:
        raise ValueError("SPARC control or write shapes disagree")
    B, L = eta.shape
    M = nu_log.numel()
    if fused_write:
        if raw_x.shape != (B, L, 2 * M):
            raise ValueError("fused SPARC write expects raw_x [B,L,2M]")
        br, bi = _fused_write(raw_x, nu_log)
    elif br.shape != (B, L, M) or bi.shape != br.shape:
        raise ValueError("SPARC control or write shapes disagree")
    _check_chunk_options(L, chunk_size, mode_block_size, backward_chunk_group, two_stage_spectral,
                         fused_output_relu, prefix_group_size, hierarchical_prefix)
    _check(eta, delta, nu_log, theta_log, br, bi)
    out_r, out_i = _run(eta, delta, nu_log, theta_log, br, bi)[0]
    if fused_output_relu:
        return torch.cat((out_r, out_i), dim=-1).relu()
    return out_r, out_i


def sparc_training_scan_dispatch(eta, delta, nu_log, theta_log, br, bi, *, chunk_size: int = 16,
                                 hierarchical_prefix: bool = False, precompute_shared: bool = False,
                                 compressed_transition: bool = False, atomic_shared: bool = False,
                                 two_stage_spectral: bool = False, compact_control_cache: bool = False,
                                 precompute_spectral: bool = False, raw_x=None, fused_write: bool = False,
                                 backward_chunk_group: int = 1, fused_output_relu: bool = False,
                                 prefix_group_size: int = 0, controller_backward_cache=None, segment_pos=None,
                                 initial_state=None, reset_first: bool = False, block_size: int = 128):
    """The reference's training entry (backward/scan.py:1754-1818): one path here for every case
    (segment resets, an initial state, a length that is not a whole number of chunks), so the
    routing reduces to its argument checks. Returns (out_r, out_i), or relu([Re h, Im h]) with
    fused_output_relu."""
    if fused_write and raw_x is None:
        raise ValueError("raw_x is required by the fused-write SPARC path")
    _no_fused_controller_backward(controller_backward_cache)
    if fused_write:
        br, bi = _fused_write(raw_x, nu_log)
    fallback = segment_pos is not None or initial_state is not None or eta.shape[1] % chunk_size != 0
    if fallback:
        out_r, out_i, _, _ = sparc_tiled_serial_scan(eta, delta, nu_log, theta_log, br, bi, segment_pos=segment_pos,
                                                     initial_state=initial_state, block_size=block_size,
                                                     reset_first=reset_first)
        if fused_output_relu:
            return torch.cat((out_r, out_i), dim=-1).relu()
        return out_r, out_i
    return sparc_chunk_scan(eta, delta, nu_log, theta_log, br, bi, chunk_size, hierarchical_prefix, precompute_shared,
                            compressed_transition, atomic_shared, two_stage_spectral, compact_control_cache,
                            precompute_spectral, mode_block_size=block_size, backward_chunk_group=backward_chunk_group,
                            fused_output_relu=fused_output_relu, prefix_group_size=prefix_group_size)


def sparc_scan_precomputed_decay(eta, delta, nu_log, theta_log, br, bi):
    """The reference's variant of sparc_scan that precomputes rho = exp(-nu e^eta) per
    (token, mode) before its serial kernel (backward/scan.py:1073-1121, 1690-1700): the same
    scan and gradients, so the same path here."""
    return sparc_scan(eta, delta, nu_log, theta_log, br, bi)
