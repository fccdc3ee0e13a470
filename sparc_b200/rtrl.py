"""RTRL online training of the SPARC cell on B200: the torch counterpart of the JAX
``SPARCRTRLCell`` (sparc-impl/sparc/layers.py:61-85) over ``stored_rtrl_step``
(training/rtrl.py:61-155).

The carry is (state, traces): the state a complex64 [B, M] tensor, the traces a dict of complex64
tensors, one per recurrent parameter (modal [B, M], content [B, W, M], controllers
[B, W+1, M]), as ``initialize_carry`` (rtrl.py:25-46) makes them. One call advances state and
traces by one step in ``rtrl_step_kernel`` and returns (next_carry, output) with
output = relu([Re h', Im h']) (or linear). As in the JAX custom VJP, the next carry carries no
gradient, a loss on the output gives every recurrent parameter the gradient
Re(cotangent * trace) from the NEW traces (``rtrl_grad_kernel``), and the input gets the one-step
gradient. The content products x content_{real,imag} and the controller projections are matrix
products here (weights detached: their gradients come from the traces)."""
from __future__ import annotations

import ctypes
import math

import torch
from torch import nn

from . import _lib

MODAL_NAMES = ("decay_log", "frequency_log", "write_log_gain", "write_phase_response",
               "write_retention_response")  # recurrence.py:5-11
CONTENT_NAMES = ("content_real", "content_imag")
CONTROLLER_NAMES = ("phase_controller", "retention_controller")
TRACE_NAMES = MODAL_NAMES + CONTENT_NAMES + CONTROLLER_NAMES


def initialize_traces(batch_size: int, input_size: int, modes: int, dtype=torch.complex64, device=None):
    """Zero traces, rtrl.py:25-41."""
    tr = {n: torch.zeros((batch_size, modes), dtype=dtype, device=device) for n in MODAL_NAMES}
    tr.update({n: torch.zeros((batch_size, input_size, modes), dtype=dtype, device=device)
               for n in CONTENT_NAMES})
    tr.update({n: torch.zeros((batch_size, input_size + 1, modes), dtype=dtype, device=device)
               for n in CONTROLLER_NAMES})
    return tr


def initialize_carry(batch_size: int, input_size: int, modes: int, dtype=torch.complex64, device=None):
    """(zero state [B, M], zero traces), rtrl.py:44-46."""
    return (torch.zeros((batch_size, modes), dtype=dtype, device=device),
            initialize_traces(batch_size, input_size, modes, dtype, device))


def _rtrl_check(rc: int, what: str):
    if rc != _lib.OK:
        msg = _lib.lib().sparc_rtrl_last_error()
        raise RuntimeError(f"{what} failed ({_lib.ERR_NAMES.get(rc, rc)}): {msg.decode() if msg else ''}")


def _fptr(t: torch.Tensor) -> int:
    return t.data_ptr()


class _RTRLStepFunction(torch.autograd.Function):
    """One RTRL step. Inputs: u [B, 2M], p [B, 2] (differentiable, the caller's products of x),
    x [B, W], reset (uint8 [B] or None), state [B, M] complex64, content_linear, then the nine
    traces (complex64) and the nine recurrent parameters in TRACE_NAMES order. Outputs the new
    state (differentiable) and the nine new traces (not differentiable)."""

    @staticmethod
    def forward(ctx, u, p, x, reset, state, content_linear, *rest):
        L = _lib.lib()
        traces, params = rest[:9], rest[9:]
        B, W = x.shape
        M = state.shape[1]
        dev = x.device
        x = x.detach().float().contiguous()
        u = u.detach().float().contiguous()
        p = p.detach().float().contiguous()
        st = torch.view_as_real(state.detach().to(torch.complex64).contiguous())
        tr = [torch.view_as_real(t.detach().to(torch.complex64).contiguous()) for t in traces]
        prm = [t.detach().float().contiguous() for t in params[:5]]
        new_state = torch.empty((B, M), dtype=torch.complex64, device=dev)
        new_tr = [torch.empty(t.shape[:-1], dtype=torch.complex64, device=dev) for t in tr]
        saved = torch.empty((B, M, L.sparc_rtrl_saved_floats()), dtype=torch.float32, device=dev)
        a = _lib.RtrlStepArgs(
            _fptr(x), _fptr(u), _fptr(p), _lib.ptr(reset), _fptr(st),
            _fptr(torch.view_as_real(new_state)), *[_fptr(t) for t in prm],
            (ctypes.c_void_p * 9)(*[_fptr(t) for t in tr]),
            (ctypes.c_void_p * 9)(*[_fptr(torch.view_as_real(t)) for t in new_tr]),
            _fptr(saved), B, W, M, int(content_linear))
        _rtrl_check(L.sparc_rtrl_step(ctypes.byref(a), _lib.stream_handle(dev)), "sparc_rtrl_step")
        ctx.save_for_backward(saved, *new_tr)
        ctx.dims = (B, W, M)
        ctx.mark_non_differentiable(*new_tr)
        ctx.set_materialize_grads(False)
        return (new_state, *new_tr)

    @staticmethod
    def backward(ctx, g_state, *g_traces):
        L = _lib.lib()
        saved, *new_tr = ctx.saved_tensors
        B, W, M = ctx.dims
        dev = saved.device
        nones = (None,) * 9
        if g_state is None:
            return (None, None, None, None, None, None) + nones + nones
        g = torch.view_as_real(g_state.to(torch.complex64).contiguous())
        grads = [torch.empty(M, dtype=torch.float32, device=dev) for _ in MODAL_NAMES]
        grads += [torch.empty((W, M), dtype=torch.float32, device=dev) for _ in CONTENT_NAMES]
        grads += [torch.empty(W + 1, dtype=torch.float32, device=dev) for _ in CONTROLLER_NAMES]
        du = torch.empty((B, 2 * M), dtype=torch.float32, device=dev)
        dp = torch.empty((B, 2), dtype=torch.float32, device=dev)
        a = _lib.RtrlGradArgs(
            _fptr(g), (ctypes.c_void_p * 9)(*[_fptr(torch.view_as_real(t)) for t in new_tr]), _fptr(saved),
            (ctypes.c_void_p * 9)(*[_fptr(t) for t in grads]), _fptr(du), _fptr(dp), B, W, M)
        _rtrl_check(L.sparc_rtrl_grad(ctypes.byref(a), _lib.stream_handle(dev)), "sparc_rtrl_grad")
        return (du, dp, None, None, None, None) + nones + tuple(grads)


def rtrl_step(params, carry, inputs: torch.Tensor, reset=None, content_activation: str = "tanh"):
    """stored_rtrl_step (rtrl.py:111-116): ((next_state, next_traces), state) for a mapping of the
    nine recurrent parameters. next_state is the state with its gradient path (the traces give
    the parameters' gradients); the returned carry is detached."""
    if content_activation not in ("tanh", "linear"):
        raise ValueError(content_activation)
    state, traces = carry
    if inputs.dim() != 2:
        raise ValueError("inputs must have shape [batch, input_size]")
    B, W = inputs.shape
    M = params["decay_log"].shape[0]
    if state.shape != (B, M):
        raise ValueError(f"state must have shape {(B, M)}")
    _lib.require_cuda(inputs, "inputs")
    x = inputs.float()
    # the content product and controller projections on the library's kernels (weights detached:
    # as in the JAX custom VJP, the parameters' gradients come from the traces)
    from .projection import _ProjectionInputs

    u, p = _ProjectionInputs.apply(x[:, None].contiguous(), params["content_real"].detach(),
                                   params["content_imag"].detach(), params["phase_controller"].detach(),
                                   params["retention_controller"].detach())
    u, p = u[:, 0], p[:, 0]
    r = None if reset is None else reset.to(device=x.device, dtype=torch.bool).to(torch.uint8).contiguous()
    out = _RTRLStepFunction.apply(u, p, x, r, state, content_activation == "linear",
                                  *[traces[n] for n in TRACE_NAMES], *[params[n] for n in TRACE_NAMES])
    new_state, new_tr = out[0], out[1:]
    next_carry = (new_state.detach(), dict(zip(TRACE_NAMES, new_tr)))
    return next_carry, new_state


# the reference's name (training/rtrl.py:111-116): (parameters, carry, inputs, reset, content_activation)
stored_rtrl_step = rtrl_step


class SPARCRTRLCell(nn.Module):
    """Torch counterpart of ``SPARCRTRLCell`` (sparc-impl/sparc/layers.py:61-85):
    ``forward(carry, inputs, reset) -> (next_carry, output)``, inputs [B, input_size]."""

    def __init__(self, input_size: int, modes: int, r_min: float = 0.0, r_max: float = 1.0,
                 max_phase: float = 6.28, content_activation: str = "tanh", output_activation: str = "relu"):
        super().__init__()
        if content_activation not in ("tanh", "linear"):
            raise ValueError(content_activation)
        if output_activation not in ("relu", "linear"):
            raise ValueError(output_activation)  # layers.py:78-81
        self.input_size = W = input_size
        self.modes = M = modes
        self.content_activation = content_activation
        self.output_activation = output_activation
        # the draws of _parameters (layers.py:17-58; initialization.py:5-39)
        frequency_log = torch.log(max_phase * torch.rand(M))
        u = torch.rand(M)
        decay_log = torch.log(-0.5 * torch.log(u * (r_max ** 2 - r_min ** 2) + r_min ** 2))
        self.frequency_log = nn.Parameter(frequency_log)
        self.decay_log = nn.Parameter(decay_log)
        self.content_real = nn.Parameter(torch.randn(W, M) / math.sqrt(2.0 * W))
        self.content_imag = nn.Parameter(torch.randn(W, M) / math.sqrt(2.0 * W))
        self.phase_controller = nn.Parameter(torch.zeros(W + 1))
        self.retention_controller = nn.Parameter(torch.zeros(W + 1))
        self.write_log_gain = nn.Parameter(torch.log(torch.sqrt(1.0 - torch.exp(-2.0 * torch.exp(decay_log)))))
        self.write_phase_response = nn.Parameter(torch.zeros(M))
        self.write_retention_response = nn.Parameter(torch.zeros(M))

    def initial_carry(self, batch_size: int, input_size: int | None = None, dtype=torch.complex64,
                      device=None):
        """(zero state, zero traces) with the reference's argument order (layers.py:84-85:
        batch_size, input_size, dtype); on the cell's device unless `device` is given."""
        if device is None:
            device = self.decay_log.device
        return initialize_carry(batch_size, self.input_size if input_size is None else input_size,
                                self.modes, dtype, device)

    def forward(self, carry, inputs: torch.Tensor, reset=None):
        if inputs.shape[-1] != self.input_size:
            raise ValueError((inputs.shape[-1], self.input_size))
        params = {n: getattr(self, n) for n in TRACE_NAMES}
        next_carry, state = rtrl_step(params, carry, inputs, reset, self.content_activation)
        output = torch.cat((state.real, state.imag), dim=-1)
        if self.output_activation == "relu":
            output = torch.relu(output)
        return next_carry, output
