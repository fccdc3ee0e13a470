"""SPARCMixer: drop-in for the reference ``sparc-kernal/sparc.py`` module on B200.

Same constructor, parameter names/shapes/initialisation (and RNG draw order), buffers,
``forward(x, return_cache=False)``, ``step(x, state, segment_pos)``, ``prepare_inference()``
and setters as sparc.py:58-123. Every call runs the sm_100a kernels of libsparc_b200 through
its C ABI; the backend setters are validated like the reference's but select nothing, since
there is exactly one code path.

Extensions over the reference module (both follow the reference's tiled serial scan,
``sparc_training_scan_dispatch`` backward/scan.py:1754-1818 -> forward/scan.py:807-854):
``forward(..., state=(h_r, h_i))`` starts the recurrence from a given state, and its gradient
flows back to that state; ``forward(..., segment_pos=pos)`` restarts the recurrence at every token
with ``pos == 0`` (packed sequences), ``reset_first=True`` at the first token when no
``segment_pos`` is given (common.py:219-268).
"""
from __future__ import annotations

import ctypes
import math

import torch
from torch import nn

from . import _lib

_PARAMS = ("nu_log", "theta_log", "phase_direction", "radial_direction", "write_log_gain",
           "energy_response", "write_phase_response", "write_radial_response")


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to(torch.float32).contiguous()


def _exchange_fields(a, device):
    """Fill the backward's fused cross-GPU gradient sum from the active exchange group of this
    device (sparc_b200.ddp.FusedGradExchange), if any."""
    from . import ddp

    ex = ddp.active_exchange(device)
    if ex is None:
        return
    for r, b in enumerate(ex.buffers):
        a.exchange_buffers[r] = b
    a.exchange_world = ex.world
    a.exchange_rank = ex.rank
    a.exchange_status = ex.status.data_ptr()


class _SparcMixerFunction(torch.autograd.Function):
    """Autograd op around sparc_mixer_forward / sparc_mixer_backward.

    Outputs y [B, T, W] (x.dtype) and the final state (last_r, last_i) [B, M] float32; both
    are differentiable. Saved for backward: x, every token's state (the forward writes them when
    a gradient can be asked for; their sign is y's relu mask), the parameters, the per-chunk
    carries and the per-token controls. With a norm weight the call is a block:
    y = x + mixer(RMSNorm(x)) in the same kernels, and the relu bits are saved as well."""

    @staticmethod
    def forward(ctx, x, nu_log, theta_log, phase_direction, radial_direction, write_log_gain,
                energy_response, write_phase_response, write_radial_response, h0_r, h0_i,
                max_spin, reset=None, norm_weight=None, norm_eps=1e-6):
        L = _lib.lib()
        B, T, W = x.shape
        M = W // 2
        dt = _lib.dtype_code(x.dtype)
        dev = x.device
        params = [_f32(p) for p in (nu_log, theta_log, phase_direction, radial_direction,
                                    write_log_gain, write_phase_response, write_radial_response)]
        h0 = None
        if h0_r is not None:
            h0 = (_f32(h0_r), _f32(h0_i))
        y = torch.empty_like(x)
        # every token's state for the backward (saves its gradient kernel the state replay);
        # only when a gradient can be asked for
        states = torch.empty_like(x) if any(ctx.needs_input_grad) else None
        block = norm_weight is not None
        nw = _f32(norm_weight) if block else None
        mask = (torch.empty((B, T, L.sparc_mixer_mask_words(W)), dtype=torch.int32, device=dev)
                if block else None)
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
            x.data_ptr(), y.data_ptr(), *[p.data_ptr() for p in params],
            _lib.ptr(h0[0] if h0 else None), _lib.ptr(h0[1] if h0 else None),
            last_r.data_ptr(), last_i.data_ptr(), carry.data_ptr(), controls.data_ptr(), _lib.ptr(reset),
            _lib.ptr(nw), float(norm_eps), _lib.ptr(mask), None, 0,
            ws.data_ptr(), ws.numel(), B, T, W, dt, max_spin, None, _lib.ptr(states))
        _lib.check(L.sparc_mixer_forward(ctypes.byref(a), _lib.stream_handle(dev)),
                   "sparc_mixer_forward")
        # the states stand in for y in the backward (their sign is y's relu mask)
        ctx.save_for_backward(x, states, *params, carry, controls, *(h0 if h0 else (None, None)), nw, mask)
        ctx.has_h0 = h0 is not None
        ctx.max_spin = max_spin
        ctx.set_materialize_grads(False)
        return y, last_r, last_i

    @staticmethod
    def backward(ctx, dy, dlast_r, dlast_i):
        L = _lib.lib()
        x, states, nu_log, theta_log, pd, rd, wlg, wpr, wrr, carry, controls, h0_r, h0_i, nw, mask = ctx.saved_tensors
        B, T, W = x.shape
        M = W // 2
        dev = x.device
        dt = _lib.dtype_code(x.dtype)
        dy = torch.zeros_like(x) if dy is None else dy.to(x.dtype).contiguous()
        if dlast_r is None and dlast_i is None:
            gl = None
        else:
            gl = (torch.zeros((B, M), device=dev) if dlast_r is None else _f32(dlast_r),
                  torch.zeros((B, M), device=dev) if dlast_i is None else _f32(dlast_i))
        dx = torch.empty_like(x)
        g = {n: torch.empty(M, dtype=torch.float32, device=dev) for n in _PARAMS}
        g["phase_direction"] = torch.empty(W + 1, dtype=torch.float32, device=dev)
        g["radial_direction"] = torch.empty(W + 1, dtype=torch.float32, device=dev)
        gnw = torch.empty(W, dtype=torch.float32, device=dev) if nw is not None else None
        gh0 = None
        if ctx.has_h0:
            gh0 = (torch.empty((B, M), dtype=torch.float32, device=dev),
                   torch.empty((B, M), dtype=torch.float32, device=dev))
        nbytes = L.sparc_mixer_workspace_bytes(B, T, W, dt)
        ws = _lib.WORKSPACES.get(dev, nbytes)
        a = _lib.MixerBwdArgs(
            x.data_ptr(), None, dy.data_ptr(), dx.data_ptr(),
            nu_log.data_ptr(), theta_log.data_ptr(), pd.data_ptr(), rd.data_ptr(),
            wlg.data_ptr(), wpr.data_ptr(), wrr.data_ptr(),
            _lib.ptr(h0_r), _lib.ptr(h0_i),
            _lib.ptr(gl[0] if gl else None), _lib.ptr(gl[1] if gl else None),
            _lib.ptr(gh0[0] if gh0 else None), _lib.ptr(gh0[1] if gh0 else None),
            carry.data_ptr(), controls.data_ptr(), _lib.ptr(nw), _lib.ptr(mask), _lib.ptr(gnw),
            *[g[n].data_ptr() for n in _PARAMS], None, 0,
            workspace=ws.data_ptr(), workspace_bytes=ws.numel(), batch=B, length=T, width=W, dtype=dt,
            max_spin=ctx.max_spin, states=_lib.ptr(states))
        _exchange_fields(a, dev)
        _lib.check(L.sparc_mixer_backward(ctypes.byref(a), _lib.stream_handle(dev)),
                   "sparc_mixer_backward")
        return (dx, *[g[n] for n in _PARAMS],
                gh0[0] if gh0 else None, gh0[1] if gh0 else None, None, None, gnw, None)


def reset_mask(segment_pos, reset_first: bool, shape, device):
    """The [B, T] byte mask of tokens whose transition is zeroed: segment_pos == 0 where
    segment_pos is given, else the first token when reset_first (common.py:219-268)."""
    B, T = shape
    if segment_pos is not None:
        if segment_pos.shape != (B, T):
            raise ValueError(f"segment_pos must have shape [batch, length] = {(B, T)}")
        return (segment_pos.to(device) == 0).to(torch.uint8).contiguous()
    if reset_first:
        m = torch.zeros((B, T), dtype=torch.uint8, device=device)
        m[:, 0] = 1
        return m
    return None


def sparc_mixer(x, params, state=None, max_spin: int = 0, segment_pos=None, reset_first: bool = False):
    """Functional form: (y, (last_r, last_i)) for parameters given as a mapping."""
    h0_r, h0_i = (None, None) if state is None else state
    reset = reset_mask(segment_pos, reset_first, x.shape[:2], x.device)
    y, lr, li = _SparcMixerFunction.apply(
        x, *[params[n] for n in _PARAMS], h0_r, h0_i, int(max_spin), reset)
    return y, (lr, li)


def sparc_block(x, params, norm_weight, eps: float = 1e-6, state=None, segment_pos=None,
                reset_first: bool = False, max_spin: int = 0):
    """One block of the config-5 stack in the mixer's own kernels: (x + mixer(RMSNorm(x)),
    (last_r, last_i)), RMSNorm(x) = x * (mean(x^2) + eps)^(-1/2) * norm_weight per token."""
    if norm_weight.shape != (x.shape[-1],):
        raise ValueError("norm_weight must have shape [width]")
    _lib.require_cuda(x, "x")
    h0_r, h0_i = (None, None) if state is None else state
    reset = reset_mask(segment_pos, reset_first, x.shape[:2], x.device)
    y, lr, li = _SparcMixerFunction.apply(
        x.contiguous(), *[params[n] for n in _PARAMS], h0_r, h0_i, int(max_spin), reset, norm_weight,
        float(eps))
    return y, (lr, li)


@torch.no_grad()
def sparc_decode_step(x: torch.Tensor, params, state):
    """One fused decode step: (y [B, W] x.dtype, (new_r, new_i) [B, M] float32)."""
    if x.dim() != 2:
        raise ValueError("decode expects x of shape [batch, width]")
    B, W = x.shape
    if W % 2:
        raise ValueError("SPARC rnn_width must be even")
    M = W // 2
    if tuple(state[0].shape) != (B, M) or tuple(state[1].shape) != (B, M):
        raise ValueError("decode state must be a pair of [batch, width/2] tensors")
    _lib.require_cuda(x, "x")
    L = _lib.lib()
    x = x.contiguous()
    dt = _lib.dtype_code(x.dtype)
    sr, si = _f32(state[0]), _f32(state[1])
    p = [_f32(params[n]) for n in ("nu_log", "theta_log", "phase_direction", "radial_direction",
                                    "write_log_gain", "write_phase_response", "write_radial_response")]
    y = torch.empty_like(x)
    nr = torch.empty((B, M), dtype=torch.float32, device=x.device)
    ni = torch.empty((B, M), dtype=torch.float32, device=x.device)
    a = _lib.DecodeArgs(x.data_ptr(), y.data_ptr(), sr.data_ptr(), si.data_ptr(), nr.data_ptr(),
                        ni.data_ptr(), *[t.data_ptr() for t in p], B, W, dt)
    _lib.check(L.sparc_decode_step(ctypes.byref(a), _lib.stream_handle(x.device)), "sparc_decode_step")
    return y, (nr, ni)


def sparc_eager_step(x: torch.Tensor, params, state):
    """The reference's decode step before ``prepare_inference()`` (forward/decode.py:296-306): one
    token of the sequence path, differentiable with respect to x, the state and every parameter.

    It runs the mixer kernels on the length-1 sequence x[:, None] with the state as the initial
    state, so its gradients are the sequence adjoint's (the write keeps float32 here, where the
    reference rounds it to x's dtype first, forward/control.py:163: with bfloat16 activations the
    two differ by that rounding, well inside the bfloat16 tolerance).
    Returns (y [B, W] x.dtype, (new_r, new_i) [B, M] float32)."""
    if x.dim() != 2:
        raise ValueError("decode expects x of shape [batch, width]")
    B, W = x.shape
    if W % 2:
        raise ValueError("SPARC rnn_width must be even")
    M = W // 2
    if tuple(state[0].shape) != (B, M) or tuple(state[1].shape) != (B, M):
        raise ValueError("decode state must be a pair of [batch, width/2] tensors")
    _lib.require_cuda(x, "x")
    y, last = sparc_mixer(x[:, None].contiguous(), params, state=(state[0], state[1]))
    return y[:, 0], last


def run_sequence(module, x: torch.Tensor, return_cache: bool = False):
    """The reference's sequence entry as a function of the module (forward/scan.py:1398-1603,
    which its SPARCMixer.forward calls): module(x, return_cache)."""
    return module(x, return_cache)


def prepare_decode(module) -> None:
    """forward/decode.py:252-255: switch the module to its fused decode step."""
    module.prepare_inference()


def run_decode_step(module, x: torch.Tensor, state, segment_pos):
    """forward/decode.py:273-306 (segment_pos is ignored there too): module.step(x, state,
    segment_pos)."""
    return module.step(x, state, segment_pos)


class SPARCMixer(nn.Module):
    """Drop-in for the reference SPARCMixer (sparc-kernal/sparc.py:58-123)."""

    def __init__(self, width: int):
        super().__init__()
        if width % 2:
            raise ValueError("SPARC rnn_width must be even")
        self.width = width
        self.modes = width // 2
        # same draws, same order and same float32 arithmetic as sparc.py:63-84
        radius_squared = torch.rand(self.modes).clamp_min(torch.finfo(torch.float32).tiny)
        nu = -0.5 * torch.log(radius_squared)
        theta = (2.0 * math.pi * torch.rand(self.modes)).clamp_min(torch.finfo(torch.float32).tiny)
        self.nu_log = nn.Parameter(torch.log(nu))
        self.theta_log = nn.Parameter(torch.log(theta))
        self.phase_direction = nn.Parameter(torch.zeros(width + 1))
        self.radial_direction = nn.Parameter(torch.zeros(width + 1))
        self.register_buffer("phase_amplitude", torch.zeros(()))
        self.register_buffer("radial_amplitude", torch.zeros(()))
        initial_gain = torch.log(torch.sqrt(1.0 - torch.exp(-2.0 * nu)) + 1.0e-8)
        self.write_log_gain = nn.Parameter(initial_gain)
        self.energy_response = nn.Parameter(torch.full((self.modes,), 0.5493061443340548))
        self.write_phase_response = nn.Parameter(torch.zeros(self.modes))
        self.write_radial_response = nn.Parameter(torch.zeros(self.modes))
        self._inference_fused = False
        self._decode_backend = "auto"
        self._inference_pack = None
        self._tiled_training_block_size = 128
        self._controller_projection_dtype = "fp32_fused_coords"
        self.scan_backend = "auto"
        self.max_spin = 0  # lookback wait bound (0 = library default)

    def _params(self):
        return {n: getattr(self, n) for n in _PARAMS}

    def forward(self, x: torch.Tensor, return_cache: bool = False, state=None, segment_pos=None,
                reset_first: bool = False):
        if x.dim() != 3 or x.shape[-1] != self.width:
            raise ValueError(f"SPARCMixer expects x of shape [batch, length, {self.width}]")
        if x.dtype not in (torch.float32, torch.bfloat16):
            raise TypeError(f"SPARCMixer supports float32 and bfloat16 activations, got {x.dtype}")
        if state is not None:
            B = x.shape[0]
            if state[0].shape != (B, self.modes) or state[1].shape != (B, self.modes):
                raise ValueError("initial SPARC states must have shape [B, M]")
        _lib.require_cuda(x, "x")
        y, cache = sparc_mixer(x.contiguous(), self._params(), state, self.max_spin,
                               segment_pos=segment_pos, reset_first=reset_first)
        return y, (cache if return_cache else None)

    # the reference's backend switches (sparc.py:93-120): validated, one code path behind them
    def set_scan_backend(self, backend: str) -> None:
        self.scan_backend = backend

    def set_tiled_training_block_size(self, block_size: int) -> None:
        if block_size not in (32, 64, 128, 256):
            raise ValueError(block_size)
        self._tiled_training_block_size = block_size

    def set_controller_projection_dtype(self, dtype: str) -> None:
        if dtype not in (
            "fp32", "bf16", "triton_fp32",
            "fp32_rounded", "triton_fp32_rounded", "fp32_recompute",
            "fp32_triton_backward", "fp32_cache_save",
            "fp32_cache_recompute", "fp32_fused_coords",
        ):
            raise ValueError(dtype)
        self._controller_projection_dtype = dtype

    def prepare_inference(self) -> None:
        self._inference_fused = True
        self._inference_pack = None

    def set_decode_backend(self, backend: str) -> None:
        if backend not in ("auto", "fused", "packed", "blocked16", "blocked32", "blocked64"):
            raise ValueError(backend)
        self._decode_backend = backend

    def step(self, x: torch.Tensor, state, segment_pos):
        """forward/decode.py:273-306: after prepare_inference() the fused decode kernel (no
        autograd, as the reference's latest_sparc_decode); before it the differentiable step."""
        del segment_pos  # ignored, as in forward/decode.py:274
        if self._inference_fused:
            return sparc_decode_step(x, self._params(), state)
        return sparc_eager_step(x, self._params(), state)
