"""The projection variant of SPARC on B200: the sequence layer of the JAX package ``sparc-impl``
(``SPARCSequenceLayer``, layers.py:88-126 over recurrence.py:20-63) as a torch module.

Unlike the torch ``SPARCMixer`` (whose content is x's two halves and whose output is
relu([Re h, Im h])), this layer writes a content u = x content_{real,imag} into M modes of any
count and reads the states out through a complex readout plus a skip:

    p = [x, 1] (phase_controller, retention_controller)        controller projections [B, T, 2]
    u = x [content_real | content_imag]                          content input [B, T, 2M]
    h = SPARC states from (u, p)                                 libsparc_b200, projection mode
    y = Re(h (readout_real + i readout_imag)^T) + skip * x

The recurrence (controls, transition, write gain, scan and their adjoints) runs in the sm_100a
kernels of libsparc_b200 in projection mode (``projections`` / ``grad_projections`` of the C
ABI); the content, projection and readout products are the layer's matrix products around it.
Parameter names and shapes are the JAX layer's; its initializers' distributions are reproduced
(initialization.py:5-39) with torch's generator, since JAX's PRNG draws cannot be.
"""
from __future__ import annotations

import ctypes
import math

import torch
from torch import nn

from . import _lib
from .mixer import reset_mask

_CORE_PARAMS = ("decay_log", "frequency_log", "write_log_gain", "write_phase_response",
                "write_retention_response")


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to(torch.float32).contiguous()


class _CoreSaved:
    """What the recurrence's backward needs from its forward."""

    def __init__(self, u, params, carry, controls, h0, lin, max_spin):
        self.u, self.params, self.carry, self.controls = u, params, carry, controls
        self.h0, self.lin, self.max_spin = h0, lin, max_spin


def _core_forward(u, p, modal, h0, reset, lin, max_spin):
    """sparc_mixer_forward in projection mode: states h [B, T, 2M] (u.dtype) and the last state
    from the content input u [B, T, 2M] and the projections p [B, T, 2] float32."""
    L = _lib.lib()
    B, T, W = u.shape
    M = W // 2
    dt = _lib.dtype_code(u.dtype)
    dev = u.device
    params = [_f32(t) for t in modal]
    p = _f32(p)
    h0 = None if h0 is None else (_f32(h0[0]), _f32(h0[1]))
    h = torch.empty_like(u)
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
        u.data_ptr(), h.data_ptr(), params[0].data_ptr(), params[1].data_ptr(), None, None,
        params[2].data_ptr(), params[3].data_ptr(), params[4].data_ptr(),
        _lib.ptr(h0[0] if h0 else None), _lib.ptr(h0[1] if h0 else None),
        last_r.data_ptr(), last_i.data_ptr(), carry.data_ptr(), controls.data_ptr(), _lib.ptr(reset),
        None, 0.0, None, p.data_ptr(), int(lin),
        ws.data_ptr(), ws.numel(), B, T, W, dt, max_spin)
    _lib.check(L.sparc_mixer_forward(ctypes.byref(a), _lib.stream_handle(dev)),
               "sparc_mixer_forward (projection mode)")
    return h, last_r, last_i, _CoreSaved(u, params, carry, controls, h0, int(lin), max_spin)


def _core_backward(sv: _CoreSaved, dh, dlast_r, dlast_i, states=None):
    """sparc_mixer_backward in projection mode: (du, dp, five modal gradients, gh0 or None).
    ``states``: the forward's output h (the states), read by the gradient kernel instead of
    replaying them."""
    L = _lib.lib()
    u = sv.u
    B, T, W = u.shape
    M = W // 2
    dev = u.device
    dt = _lib.dtype_code(u.dtype)
    dh = torch.zeros_like(u) if dh is None else dh.to(u.dtype).contiguous()
    if dlast_r is None and dlast_i is None:
        gl = None
    else:
        gl = (torch.zeros((B, M), device=dev) if dlast_r is None else _f32(dlast_r),
              torch.zeros((B, M), device=dev) if dlast_i is None else _f32(dlast_i))
    du = torch.empty_like(u)
    dp = torch.empty((B, T, 2), dtype=torch.float32, device=dev)
    g = [torch.empty(M, dtype=torch.float32, device=dev) for _ in range(6)]  # (+ energy slot)
    gh0 = None
    if sv.h0 is not None:
        gh0 = (torch.empty((B, M), dtype=torch.float32, device=dev),
               torch.empty((B, M), dtype=torch.float32, device=dev))
    dlog, flog, wlg, wpr, wrr = sv.params
    ws = _lib.WORKSPACES.get(dev, L.sparc_mixer_workspace_bytes(B, T, W, dt))
    a = _lib.MixerBwdArgs(
        u.data_ptr(), None, dh.data_ptr(), du.data_ptr(),
        dlog.data_ptr(), flog.data_ptr(), None, None, wlg.data_ptr(), wpr.data_ptr(), wrr.data_ptr(),
        _lib.ptr(sv.h0[0] if sv.h0 else None), _lib.ptr(sv.h0[1] if sv.h0 else None),
        _lib.ptr(gl[0] if gl else None), _lib.ptr(gl[1] if gl else None),
        _lib.ptr(gh0[0] if gh0 else None), _lib.ptr(gh0[1] if gh0 else None),
        sv.carry.data_ptr(), sv.controls.data_ptr(), None, None, None,
        g[0].data_ptr(), g[1].data_ptr(), None, None, g[2].data_ptr(), g[5].data_ptr(),
        g[3].data_ptr(), g[4].data_ptr(), dp.data_ptr(), sv.lin,
        workspace=ws.data_ptr(), workspace_bytes=ws.numel(), batch=B, length=T, width=W, dtype=dt,
        max_spin=sv.max_spin, states=_lib.ptr(states))
    _lib.check(L.sparc_mixer_backward(ctypes.byref(a), _lib.stream_handle(dev)),
               "sparc_mixer_backward (projection mode)")
    return du, dp, g[:5], gh0


class _SparcCoreFunction(torch.autograd.Function):
    """Autograd op around the recurrence in projection mode.

    Inputs: the content input u [B, T, 2M] (float32 or bfloat16), the controller projections
    p [B, T, 2] float32 (bias included) and the five modal parameters. Outputs the states
    h = [Re h, Im h] [B, T, 2M] (u.dtype) and the last state (last_r, last_i) [B, M] float32."""

    @staticmethod
    def forward(ctx, u, p, decay_log, frequency_log, write_log_gain, write_phase_response,
                write_retention_response, h0_r, h0_i, max_spin, reset, content_linear):
        h0 = None if h0_r is None else (h0_r, h0_i)
        h, lr, li, sv = _core_forward(u, p, (decay_log, frequency_log, write_log_gain, write_phase_response,
                                             write_retention_response), h0, reset, content_linear, max_spin)
        ctx.sv = sv
        ctx.save_for_backward(h)
        ctx.set_materialize_grads(False)
        return h, lr, li

    @staticmethod
    def backward(ctx, dh, dlast_r, dlast_i):
        (h,) = ctx.saved_tensors
        du, dp, g, gh0 = _core_backward(ctx.sv, dh, dlast_r, dlast_i, states=h)
        ctx.sv = None
        return (du, dp, *g, gh0[0] if gh0 else None, gh0[1] if gh0 else None, None, None, None)


class _SequenceLayerTC(torch.autograd.Function):
    """The whole layer on the library's kernels: the controller projections p = [x, 1] c
    (sparc_proj_rowdot), the content product u = x Wc and the readout on the tensor cores
    (sparc_proj_gemm, tcgen05) around the recurrence (the mixer kernels' projection mode); in the
    backward dh = dy Ro, dx = du Wc^T + dp c^T + skip dy and the weight gradients x^T du and
    dy^T h on the tensor cores (the last two with the token-major operands as stored), and the
    controllers' and skip's gradients as column sums (sparc_proj_colsum). bfloat16 activations:
    bf16 operands, the skip and rank-2 terms fused into the products' epilogues. float32
    activations: each product through the three-term bf16 split (gemm.split3, relative error
    ~1e-5), the skip terms as adds. Widths that are not multiples of 8 are zero-padded to whole
    16-byte rows for the tensor maps (the padding contributes zeros and is cut from the results)."""

    @staticmethod
    def forward(ctx, x, content_real, content_imag, phase_controller, retention_controller, decay_log,
                frequency_log, write_log_gain, write_phase_response, write_retention_response, readout_real,
                readout_imag, skip, h0_r, h0_i, reset, lin, max_spin):
        from . import gemm

        B, T, W = x.shape
        M = content_real.shape[1]
        f32 = x.dtype == torch.float32
        xf = x.reshape(B * T, W)
        xp = gemm.pad8(xf)                                                          # [BT, W8]
        wc = torch.cat((content_real, content_imag), dim=1).detach().float()       # [W, 2M]
        ro = torch.cat((readout_real, -readout_imag), dim=1).detach().float()      # [W, 2M]
        ctl = torch.stack((phase_controller, retention_controller), dim=1).detach().float()  # [W+1, 2]
        p = gemm.proj_rowdot(xf, ctl).view(B, T, 2)
        wct = gemm.pad8(wc.t().contiguous())                                       # [2M, W8]
        if f32:
            u = gemm.proj_gemm_f32(xp, wct).view(B, T, 2 * M)
        else:
            u = gemm.proj_gemm(xp, wct.to(torch.bfloat16).contiguous()).view(B, T, 2 * M)
        h0 = None if h0_r is None else (h0_r, h0_i)
        h, lr, li, sv = _core_forward(u, p, (decay_log, frequency_log, write_log_gain, write_phase_response,
                                             write_retention_response), h0, reset, lin, max_spin)
        skipf = skip.detach().float()
        hp = gemm.pad8(h.view(B * T, 2 * M))                                       # [BT, 2M8]
        rop = gemm.pad8(ro)                                                        # [W, 2M8]
        if f32:
            y = torch.addcmul(gemm.proj_gemm_f32(hp, rop), skipf, xf).view(B, T, W)
        else:
            y = gemm.proj_gemm(hp, rop.to(torch.bfloat16).contiguous(), x=xf, skip=skipf).view(B, T, W)
        ctx.sv = sv
        ctx.save_for_backward(x, h, wc, ro, ctl, skipf)
        ctx.set_materialize_grads(False)
        return y, lr, li

    @staticmethod
    def backward(ctx, dy, dlast_r, dlast_i):
        from . import gemm

        x, h, wc, ro, ctl, skip = ctx.saved_tensors
        B, T, W = x.shape
        M2 = h.shape[-1]
        f32 = x.dtype == torch.float32
        xf = x.reshape(B * T, W)
        hf = h.reshape(B * T, M2)
        dyf = None if dy is None else dy.to(x.dtype).reshape(B * T, W).contiguous()
        dh = None
        if dyf is not None:
            dyp = gemm.pad8(dyf)                                                   # [BT, W8]
            rot = gemm.pad8(ro.t().contiguous())                                   # [2M, W8]
            if f32:
                dh = gemm.proj_gemm_f32(dyp, rot).view(B, T, M2)
            else:
                dh = gemm.proj_gemm(dyp, rot.to(torch.bfloat16).contiguous()).view(B, T, M2)
        du, dp, g, gh0 = _core_backward(ctx.sv, dh, dlast_r, dlast_i, states=h)
        ctx.sv = None
        du2 = du.view(B * T, M2)
        dp2 = dp.view(B * T, 2)
        dup = gemm.pad8(du2)                                                       # [BT, 2M8]
        wcp = gemm.pad8(wc)                                                        # [W, 2M8]
        c0, c1 = ctl[:W, 0].contiguous(), ctl[:W, 1].contiguous()
        if f32:
            dx = gemm.proj_gemm_f32(dup, wcp, dp=dp2, c0=c0, c1=c1)
            if dyf is not None:
                dx = torch.addcmul(dx, skip, dyf)
        elif dyf is not None:
            dx = gemm.proj_gemm(dup, wcp.to(torch.bfloat16).contiguous(), x=dyf, skip=skip, dp=dp2, c0=c0, c1=c1)
        else:
            dx = gemm.proj_gemm(dup, wcp.to(torch.bfloat16).contiguous(), dp=dp2, c0=c0, c1=c1)
        # weight gradients over the tokens, the operands token-major as stored: x^T du, dy^T h
        xp = gemm.pad8(xf)
        prod = gemm.proj_gemm_f32 if f32 else (lambda a, b, **kw: gemm.proj_gemm(a, b, torch.float32, **kw))
        dwc = prod(xp, dup, a_mn=True, b_mn=True)[:W, :M2]                        # [W, 2M]
        if dyf is not None:
            dro = prod(dyp, gemm.pad8(hf), a_mn=True, b_mn=True)[:W, :M2]
        else:
            dro = torch.zeros((W, M2), dtype=torch.float32, device=x.device)
        dctl, dskip = gemm.proj_colsum(xf, dp2, dyf)
        if dskip is None:
            dskip = torch.zeros(W, dtype=torch.float32, device=x.device)
        M = M2 // 2
        return (dx.view(B, T, W), dwc[:, :M], dwc[:, M:], dctl[:, 0], dctl[:, 1], *g, dro[:, :M], -dro[:, M:],
                dskip, gh0[0] if gh0 else None, gh0[1] if gh0 else None, None, None, None)


def _check_activation(content_activation: str) -> bool:
    if content_activation not in ("tanh", "linear"):
        raise ValueError(content_activation)  # recurrence.py:41-48
    return content_activation == "linear"


class _ProjectionInputs(torch.autograd.Function):
    """(u [B, T, 2M] x.dtype, p [B, T, 2] float32) = (x [content_real | content_imag],
    [x, 1] [phase_controller | retention_controller]) on the library's kernels (tcgen05 product,
    row dots), with their adjoints (dx = du Wc^T + dp c^T, x^T du token-major, column sums)."""

    @staticmethod
    def forward(ctx, x, content_real, content_imag, phase_controller, retention_controller):
        from . import gemm

        B, T, W = x.shape
        M = content_real.shape[1]
        xf = x.reshape(B * T, W)
        wc = torch.cat((content_real, content_imag), dim=1).detach().float()       # [W, 2M]
        ctl = torch.stack((phase_controller, retention_controller), dim=1).detach().float()
        p = gemm.proj_rowdot(xf, ctl).view(B, T, 2)
        wct = gemm.pad8(wc.t().contiguous())
        if x.dtype == torch.float32:
            u = gemm.proj_gemm_f32(gemm.pad8(xf), wct).view(B, T, 2 * M)
        else:
            u = gemm.proj_gemm(gemm.pad8(xf), wct.to(torch.bfloat16).contiguous()).view(B, T, 2 * M)
        ctx.save_for_backward(x, wc, ctl)
        ctx.set_materialize_grads(False)
        return u, p

    @staticmethod
    def backward(ctx, du, dp):
        from . import gemm

        x, wc, ctl = ctx.saved_tensors
        B, T, W = x.shape
        M2 = wc.shape[1]
        M = M2 // 2
        f32 = x.dtype == torch.float32
        xf = x.reshape(B * T, W)
        du2 = torch.zeros((B * T, M2), dtype=x.dtype, device=x.device) if du is None else \
            du.to(x.dtype).reshape(B * T, M2).contiguous()
        dp2 = torch.zeros((B * T, 2), dtype=torch.float32, device=x.device) if dp is None else \
            dp.float().reshape(B * T, 2).contiguous()
        dup, wcp = gemm.pad8(du2), gemm.pad8(wc)
        c0, c1 = ctl[:W, 0].contiguous(), ctl[:W, 1].contiguous()
        need = ctx.needs_input_grad
        dx = dwc = dctl = None
        if need[0]:
            if f32:
                dx = gemm.proj_gemm_f32(dup, wcp, dp=dp2, c0=c0, c1=c1).view(B, T, W)
            else:
                dx = gemm.proj_gemm(dup, wcp.to(torch.bfloat16).contiguous(), dp=dp2, c0=c0, c1=c1).view(B, T, W)
        if need[1] or need[2]:
            if f32:
                dwc = gemm.proj_gemm_f32(gemm.pad8(xf), dup, a_mn=True, b_mn=True)[:W, :M2]
            else:
                dwc = gemm.proj_gemm(gemm.pad8(xf), dup, torch.float32, a_mn=True, b_mn=True)[:W, :M2]
        if need[3] or need[4]:
            dctl, _ = gemm.proj_colsum(xf, dp2)
        return (dx, None if dwc is None else dwc[:, :M], None if dwc is None else dwc[:, M:],
                None if dctl is None else dctl[:, 0], None if dctl is None else dctl[:, 1])


def sparc_projection_states(x, params, content_activation: str = "tanh", state=None, segment_pos=None,
                            reset_first: bool = False, max_spin: int = 0):
    """The recurrent core of the projection variant: ((h_r, h_i) [B, T, M] each in x.dtype,
    (last_r, last_i) [B, M] float32) for x [B, T, W] and a mapping holding the JAX layer's
    recurrent parameters (content_real/imag [W, M], the two controllers [W+1], the five modal
    vectors [M]); differentiable in x and every parameter."""
    lin = _check_activation(content_activation)
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"supported activations are float32 and bfloat16, got {x.dtype}")
    _lib.require_cuda(x, "x")
    M = params["decay_log"].shape[0]
    u, p = _ProjectionInputs.apply(x.contiguous(), params["content_real"], params["content_imag"],
                                   params["phase_controller"], params["retention_controller"])
    h0_r, h0_i = (None, None) if state is None else state
    reset = reset_mask(segment_pos, reset_first, x.shape[:2], x.device)
    h, lr, li = _SparcCoreFunction.apply(
        u, p, *[params[n] for n in _CORE_PARAMS], h0_r, h0_i, int(max_spin), reset, lin)
    return (h[..., :M], h[..., M:]), (lr, li)


def sparc_sequence_layer(x, params, content_activation: str = "tanh", state=None, segment_pos=None,
                         reset_first: bool = False, max_spin: int = 0):
    """Functional SPARCSequenceLayer: (y [B, T, W], (last_r, last_i)), every product and the
    recurrence in the library's kernels (_SequenceLayerTC)."""
    lin = _check_activation(content_activation)
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"supported activations are float32 and bfloat16, got {x.dtype}")
    _lib.require_cuda(x, "x")
    h0_r, h0_i = (None, None) if state is None else state
    reset = reset_mask(segment_pos, reset_first, x.shape[:2], x.device)
    y, lr, li = _SequenceLayerTC.apply(
        x.contiguous(), params["content_real"], params["content_imag"], params["phase_controller"],
        params["retention_controller"], *[params[n] for n in _CORE_PARAMS], params["readout_real"],
        params["readout_imag"], params["skip"], h0_r, h0_i, reset, lin, int(max_spin))
    return y, (lr, li)


class SPARCSequenceLayer(nn.Module):
    """Torch counterpart of ``SPARCSequenceLayer`` (sparc-impl/sparc/layers.py:88-126).

    ``forward(x)`` returns y [B, T, model_width] like the JAX layer's ``__call__``; the optional
    ``state`` / ``segment_pos`` / ``reset_first`` / ``return_cache`` arguments mirror
    ``SPARCMixer.forward`` (initial state with gradient, packed-sequence resets, last state)."""

    def __init__(self, model_width: int, modes: int, r_min: float = 0.9, r_max: float = 0.999,
                 max_phase: float = 6.28, content_activation: str = "tanh"):
        super().__init__()
        _check_activation(content_activation)
        self.model_width = W = model_width
        self.modes = M = modes
        self.content_activation = content_activation
        self.max_spin = 0
        # draw order of _parameters (layers.py:17-58), then the readout and skip (layers.py:112-124)
        u = torch.rand(M)
        frequency_log = torch.log(max_phase * u)
        u = torch.rand(M)
        decay_log = torch.log(-0.5 * torch.log(u * (r_max ** 2 - r_min ** 2) + r_min ** 2))
        self.frequency_log = nn.Parameter(frequency_log)
        self.decay_log = nn.Parameter(decay_log)
        self.content_real = nn.Parameter(torch.randn(W, M) / math.sqrt(2.0 * W))
        self.content_imag = nn.Parameter(torch.randn(W, M) / math.sqrt(2.0 * W))
        self.phase_controller = nn.Parameter(torch.zeros(W + 1))
        self.retention_controller = nn.Parameter(torch.zeros(W + 1))
        # write_log_gain_initializer: log sqrt(1 - |exp(-nu + i theta)|^2)
        self.write_log_gain = nn.Parameter(torch.log(torch.sqrt(1.0 - torch.exp(-2.0 * torch.exp(decay_log)))))
        self.write_phase_response = nn.Parameter(torch.zeros(M))
        self.write_retention_response = nn.Parameter(torch.zeros(M))
        self.readout_real = nn.Parameter(torch.randn(W, M) / math.sqrt(M))
        self.readout_imag = nn.Parameter(torch.randn(W, M) / math.sqrt(M))
        self.skip = nn.Parameter(torch.randn(W))

    def parameters_dict(self):
        return {n: getattr(self, n) for n, _ in self.named_parameters()}

    def forward(self, x: torch.Tensor, state=None, segment_pos=None, reset_first: bool = False,
                return_cache: bool = False):
        if x.shape[-1] != self.model_width:
            raise ValueError((x.shape[-1], self.model_width))  # layers.py:98-99
        if x.dim() != 3:
            raise ValueError("SPARCSequenceLayer expects x of shape [batch, length, model_width]")
        y, last = sparc_sequence_layer(x.contiguous(), self.parameters_dict(), self.content_activation,
                                       state, segment_pos, reset_first, self.max_spin)
        return (y, last) if return_cache else y
