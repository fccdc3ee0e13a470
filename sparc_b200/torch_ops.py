"""PyTorch operators over the libsparc_b200 C ABI: ``torch.ops.sparc_b200.mixer_forward``,
``mixer_backward``, ``decode_step``, ``real_scan_forward`` and ``real_scan_backward``
(registered by csrc_torch/torch_ops.cpp with TORCH_LIBRARY, CUDA dispatch key). They take and
return CUDA tensors and run on PyTorch's current stream; `load()` makes them available.

`load()` also registers, for every operator, a fake kernel (output shapes and dtypes from the
library's host-only queries, symbolic lengths included), so that torch.compile / make_fx can
trace calls to them, and autograd formulas for ``mixer_forward`` (through ``mixer_backward``)
and ``real_scan_forward`` (through ``real_scan_backward``): their first output is
differentiable with respect to the activations and parameters; the saved carries, controls,
states and last states are marked non-differentiable."""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib

TORCH_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libsparc_b200_torch.so")
_loaded = False


def _registered() -> bool:
    try:
        torch.ops.sparc_b200.mixer_forward
        return True
    except (AttributeError, RuntimeError):
        return False


def load():
    """Load the operator library (its C-ABI symbols resolve against libsparc_b200.so, opened here
    with global visibility first); returns torch.ops.sparc_b200."""
    global _loaded
    if not _loaded and _registered():  # (already registered in this process, e.g. by the builder)
        _loaded = True
    if not _loaded:
        if not os.path.exists(TORCH_LIB_PATH):
            raise RuntimeError(f"{TORCH_LIB_PATH} is missing: run `python -m sparc_b200._build --torch`")
        ctypes.CDLL(_lib.LIB_PATH, mode=ctypes.RTLD_GLOBAL)
        torch.ops.load_library(TORCH_LIB_PATH)
        _loaded = True
    _register_python_kernels()
    return torch.ops.sparc_b200


_python_kernels = False
_MIXER_PARAMS = 7  # nu_log, theta_log, phase/radial direction, write_log_gain, write phase/radial response


def _ceil_div(n, d: int):
    return (n + d - 1) // d  # (also for symbolic n)


def _register_python_kernels():
    """Fake kernels and autograd formulas of the operators (once per process)."""
    global _python_kernels
    if _python_kernels:
        return
    _python_kernels = True
    L = _lib.lib()
    f32 = torch.float32

    @torch.library.register_fake("sparc_b200::mixer_forward")
    def _(x, nu_log, theta_log, phase_direction, radial_direction, write_log_gain, write_phase_response,
          write_radial_response):
        B, T, W = x.shape
        M = W // 2
        chunk = L.sparc_mixer_chunk_tokens(_lib.dtype_code(x.dtype))
        return (torch.empty_like(x, memory_format=torch.contiguous_format), x.new_empty((B, M), dtype=f32),
                x.new_empty((B, M), dtype=f32), x.new_empty((B, _ceil_div(T, chunk), M, 2), dtype=f32),
                x.new_empty((B, T, L.sparc_mixer_controls_floats()), dtype=f32),
                torch.empty_like(x, memory_format=torch.contiguous_format))

    @torch.library.register_fake("sparc_b200::mixer_backward")
    def _(x, y, dy, nu_log, theta_log, phase_direction, radial_direction, write_log_gain, write_phase_response,
          write_radial_response, carry, controls, states=None):
        W = x.shape[2]
        M = W // 2
        sizes = (M, M, W + 1, W + 1, M, M, M, M)  # energy_response's (zero) gradient sixth
        return [torch.empty_like(x, memory_format=torch.contiguous_format)] + [x.new_empty((n,), dtype=f32)
                                                                               for n in sizes]

    @torch.library.register_fake("sparc_b200::decode_step")
    def _(x, state_r, state_i, nu_log, theta_log, phase_direction, radial_direction, write_log_gain,
          write_phase_response, write_radial_response):
        B, W = x.shape
        return (torch.empty_like(x, memory_format=torch.contiguous_format), x.new_empty((B, W // 2), dtype=f32),
                x.new_empty((B, W // 2), dtype=f32))

    @torch.library.register_fake("sparc_b200::real_scan_forward")
    def _(a, b):
        B, T, D = a.shape
        return (torch.empty_like(b, memory_format=torch.contiguous_format),
                a.new_empty((B, _ceil_div(T, L.sparc_real_chunk_tokens()), D), dtype=f32),
                a.new_empty((B, D), dtype=f32))

    @torch.library.register_fake("sparc_b200::real_scan_backward")
    def _(a, b, grad_out, carry):
        return (torch.empty_like(a, memory_format=torch.contiguous_format),
                torch.empty_like(b, memory_format=torch.contiguous_format))

    def mixer_setup(ctx, inputs, output):
        y, last_r, last_i, carry, controls, states = output
        ctx.mark_non_differentiable(last_r, last_i, carry, controls, states)
        ctx.save_for_backward(inputs[0], y, *inputs[1:], carry, controls, states)
        ctx.dtypes = [t.dtype for t in inputs]

    def mixer_backward(ctx, gy, g_last_r, g_last_i, g_carry, g_controls, g_states):
        x, y, *rest = ctx.saved_tensors
        params, carry, controls = rest[:_MIXER_PARAMS], rest[_MIXER_PARAMS], rest[_MIXER_PARAMS + 1]
        states = rest[_MIXER_PARAMS + 2]
        g = torch.ops.sparc_b200.mixer_backward(x, y, gy, *params, carry, controls, states)
        grads = [g[0]] + g[1:6] + g[7:9]  # (the operator takes no energy_response)
        return tuple(t.to(d) for t, d in zip(grads, ctx.dtypes))

    torch.library.register_autograd("sparc_b200::mixer_forward", mixer_backward, setup_context=mixer_setup)

    def real_setup(ctx, inputs, output):
        out, carry, last = output
        ctx.mark_non_differentiable(carry, last)
        ctx.save_for_backward(inputs[0], inputs[1], carry)
        ctx.dtypes = (inputs[0].dtype, inputs[1].dtype)

    def real_backward(ctx, g_out, g_carry, g_last):
        a, b, carry = ctx.saved_tensors
        ga, gb = torch.ops.sparc_b200.real_scan_backward(a, b, g_out, carry)
        return ga.to(ctx.dtypes[0]), gb.to(ctx.dtypes[1])

    torch.library.register_autograd("sparc_b200::real_scan_forward", real_backward, setup_context=real_setup)
