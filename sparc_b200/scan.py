"""Scan-level functional entry points of the reference module: the SPARC recurrence from
precomputed per-token controls (eta, delta) [B, L] and writes (br, bi) [B, L, M], as
``sparc_scan``, ``sparc_chunk_scan``, ``sparc_scan_with_last``, ``sparc_tiled_serial_scan``,
``sparc_training_scan_dispatch`` and ``sparc_scan_precomputed_decay``
(sparc-kernal/backward/scan.py:1658-1877, re-exported by sparc.py:17-29):

    rho = exp(-nu e^eta),  phi = theta + (1 - rho) delta,  h_t = rho e^{i phi} h_{t-1} + b_t
    (nu = e^{nu_log}, theta = e^{theta_log}; forward/scan.py:725-757).

They run the mixer's projection-mode kernels (the ones behind SPARCSequenceLayer) through a
change of variables, with no kernel of their own. Those kernels take per-token controller
projections p and a content input u and form eta' = ln16 tanh(p1), delta' = (pi/2) tanh(p0) and
the write gain(u) = e^{wlg} sqrt(expm1(-2 nu e^eta') / expm1(-2 nu)) 2 sigma(tau0 wpr + tau1 wrr) u.
With p = (atanh(delta / (pi/2)), atanh(eta / ln16)), wlg = wpr = wrr = 0 and a linear content
u = b / sqrt(expm1(-2 nu e^eta) / expm1(-2 nu)), they compute exactly the scan above, and
autograd through the change of variables gives the gradients of eta, delta, the writes,
nu_log, theta_log and the initial state.

Domain: |eta| < ln 16 and |delta| < pi/2, the range of the reference's controller
(forward/control.py:129-139: eta = ln16 tanh(p1), delta = (pi/2) tanh(p0)); values at or beyond
it are clamped to (1 - 2^-23) times the bound (and get no gradient there); the writes stay b.
"""
from __future__ import annotations

import math

import torch

from . import _lib

LN16 = math.log(16.0)
HALF_PI = 0.5 * math.pi
_EDGE = 1.0 - 2.0 ** -23  # a float32 just below 1, where atanh is still finite (about 8.3)


def _io_dtype(dtype: torch.dtype) -> torch.dtype:
    return dtype if dtype in (torch.float32, torch.bfloat16) else torch.float32


def _projection_inputs(eta, delta, nu_log, br, bi):
    """(u [B, L, 2M], p [B, L, 2] float32): the content input and controller projections for
    which the projection-mode kernels compute the scan with controls (eta, delta) and writes
    (br, bi). Differentiable in every argument."""
    x0 = (delta.float() / HALF_PI).clamp(-_EDGE, _EDGE)  # tanh(p0), tanh(p1) as the kernels will form them
    x1 = (eta.float() / LN16).clamp(-_EDGE, _EDGE)
    p = torch.stack((torch.atanh(x0), torch.atanh(x1)), dim=-1)
    nu = torch.exp(nu_log.float())
    z = nu * torch.exp(LN16 * x1)[..., None]  # (the clamped eta, so the writes are b also at the bound)
    s = torch.sqrt(torch.expm1(-2.0 * z) / torch.expm1(-2.0 * nu))
    u = torch.cat((br.float() / s, bi.float() / s), dim=-1).to(_io_dtype(br.dtype))
    return u, p


def _core(u, p, nu_log, theta_log, h0, reset):
    """The projection-mode recurrence (sparc_mixer_forward / _backward through
    projection._SparcCoreFunction): (h [B, L, 2M], last_r, last_i)."""
    from .projection import _SparcCoreFunction

    _lib.require_cuda(u, "the writes")
    zeros = torch.zeros_like(nu_log, dtype=torch.float32)
    h0_r, h0_i = (None, None) if h0 is None else h0
    return _SparcCoreFunction.apply(u, p, nu_log, theta_log, zeros, zeros, zeros, h0_r, h0_i, 0, reset, True)


def _run(eta, delta, nu_log, theta_log, br, bi, h0=None, reset=None):
    """(out_r, out_i) in br's dtype and (last_r, last_i) float32."""
    M = br.shape[-1]
    u, p = _projection_inputs(eta, delta, nu_log, br, bi)
    h, last_r, last_i = _core(u, p, nu_log, theta_log, h0, reset)
    return (h[..., :M].to(br.dtype).contiguous(), h[..., M:].to(bi.dtype).contiguous()), (last_r, last_i)


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
