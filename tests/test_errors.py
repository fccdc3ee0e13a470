"""Error behaviour of the boundary, without a GPU.

* The Python API raises ValueError for bad shapes before it looks at the device, as the
  reference's autograd functions do (backward/scan.py:796-797, 828-832, 1138-1148,
  sparc.py:61-62, 96-120); a well-shaped CPU tensor then fails loudly (no CPU path).
* Every C-ABI entry point rejects null, inconsistent or out-of-range arguments with the
  documented SPARC_ERR_* code and a message, before any device work. Every case below is
  rejected by the host-side checks: no pointer passed here is ever dereferenced or launched on.
"""
import ctypes

import pytest
import torch

import sparc_b200
from sparc_b200 import _lib

ARG, SHAPE, DTYPE, WORKSPACE = -1, -2, -3, -4
FAKE = 0x100000  # a 16-byte aligned address that the checks reject before any use


@pytest.fixture(scope="module")
def L():
    from sparc_b200 import _build

    _build.build()
    return _lib.load_library()


def _msg(fn):
    m = fn()
    return m.decode() if m else ""


# ------------------------------------------------------------------ Python API (shape first)

def test_mixer_shape_errors_precede_the_device_check():
    torch.manual_seed(0)
    m = sparc_b200.SPARCMixer(8)
    with pytest.raises(ValueError, match="rnn_width must be even"):
        sparc_b200.SPARCMixer(9)
    with pytest.raises(ValueError, match="batch, length, 8"):
        m(torch.randn(2, 3, 6))
    with pytest.raises(ValueError, match="batch, length, 8"):
        m(torch.randn(3, 8))
    with pytest.raises(TypeError):
        m(torch.randn(2, 3, 8, dtype=torch.float64))
    with pytest.raises(ValueError, match=r"\[B, M\]"):
        m(torch.randn(2, 3, 8), state=(torch.zeros(2, 3), torch.zeros(2, 4)))
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.randn(2, 3, 8))


def test_decode_shape_errors_precede_the_device_check():
    m = sparc_b200.SPARCMixer(8)
    st = (torch.zeros(2, 4), torch.zeros(2, 4))
    with pytest.raises(ValueError, match=r"\[batch, width\]"):
        m.step(torch.randn(2, 1, 8), st, None)
    with pytest.raises(ValueError, match="even"):
        sparc_b200.sparc_decode_step(torch.randn(2, 7), m._params(), st)
    with pytest.raises(ValueError, match="state"):
        m.step(torch.randn(2, 8), (torch.zeros(2, 4), torch.zeros(3, 4)), None)
    with pytest.raises(RuntimeError, match="CUDA"):
        m.step(torch.randn(2, 8), st, None)


def test_real_scan_shape_errors_precede_the_device_check():
    a, b = torch.rand(2, 32, 3), torch.rand(2, 32, 3)
    with pytest.raises(ValueError, match=r"matching \[B, L, D\]"):
        sparc_b200.real_scan(a, b[:, :16])
    with pytest.raises(ValueError, match=r"matching \[B, L, D\]"):
        sparc_b200.real_scan(a[0], b[0])
    with pytest.raises(ValueError, match=r"matching \[B, L, D\]"):
        sparc_b200.real_scan_with_last(a, b[..., :2])
    for c in (8, 48):
        with pytest.raises(ValueError, match="chunk size"):
            sparc_b200.real_chunk_scan(a, b, c)
    with pytest.raises(ValueError, match="chunk size"):
        sparc_b200.real_chunk_scan(a[:, :24], b[:, :24], 16)  # 16 does not divide 24
    with pytest.raises(RuntimeError, match="CUDA"):
        sparc_b200.real_chunk_scan(a, b, 16)


def test_projection_and_rtrl_errors_precede_the_device_check():
    torch.manual_seed(0)
    layer = sparc_b200.SPARCSequenceLayer(8, 4)
    with pytest.raises(ValueError):
        layer(torch.randn(2, 3, 6))
    with pytest.raises(ValueError):
        sparc_b200.SPARCSequenceLayer(8, 4, content_activation="relu")(torch.randn(2, 3, 8))
    with pytest.raises(RuntimeError, match="CUDA"):
        layer(torch.randn(2, 3, 8))
    cell = sparc_b200.SPARCRTRLCell(6, 4)
    carry = cell.initial_carry(2)
    with pytest.raises(ValueError):
        cell(carry, torch.randn(2, 5))
    with pytest.raises(ValueError, match="state"):
        cell(cell.initial_carry(3), torch.randn(2, 6))
    with pytest.raises(RuntimeError, match="CUDA"):
        cell(carry, torch.randn(2, 6))


def test_gemm_operand_errors_precede_the_device_check():
    from sparc_b200 import gemm

    a = torch.randn(4, 8).bfloat16()
    with pytest.raises(TypeError, match="bfloat16"):
        gemm.proj_gemm(a.float(), a)
    with pytest.raises(ValueError, match="contraction lengths"):
        gemm.proj_gemm(a, a[:, :4])
    with pytest.raises(ValueError, match="contraction lengths"):
        gemm.proj_gemm(a, a, a_mn=True)  # a [k=4, rows=8] against b [n=4, k=8]
    with pytest.raises(ValueError, match="two matrices"):
        gemm.proj_gemm(a[0], a)
    with pytest.raises(RuntimeError, match="CUDA"):
        gemm.proj_gemm(a, a)


# ------------------------------------------------------------------ C ABI

def _mixer_fwd(**kw):
    a = _lib.MixerFwdArgs(*([FAKE] * 9), None, None, FAKE, FAKE, FAKE, FAKE, None, None, 0.0, None, None, 0,
                          workspace=FAKE, workspace_bytes=1 << 30, batch=2, length=16, width=8,
                          dtype=_lib.DTYPE_F32, max_spin=0)
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def _mixer_bwd(**kw):
    a = _lib.MixerBwdArgs(*([FAKE] * 11), *([None] * 6), FAKE, FAKE, None, None, None, *([FAKE] * 8), None, 0,
                          workspace=FAKE, workspace_bytes=1 << 30, batch=2, length=16, width=8,
                          dtype=_lib.DTYPE_F32, max_spin=0)
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("change,code,words", [
    (dict(batch=0), SHAPE, "positive"),
    (dict(length=-1), SHAPE, "positive"),
    (dict(width=7), SHAPE, "even"),
    (dict(width=4098), SHAPE, "4096"),
    (dict(dtype=5), DTYPE, "dtype"),
    (dict(batch=70000, length=1, width=2), SHAPE, "carry scan"),
    (dict(norm_weight=FAKE, projections=FAKE), ARG, "exclude"),
])
def test_mixer_forward_rejects(L, change, code, words):
    for fn in (L.sparc_mixer_forward, L.sparc_mixer_forward_noalloc):
        assert fn(ctypes.byref(_mixer_fwd(**change)), None) == code
        assert words in _msg(L.sparc_last_error)


@pytest.mark.parametrize("change,code,words", [
    (dict(batch=0), SHAPE, "positive"),
    (dict(width=9), SHAPE, "even"),
    (dict(dtype=-1), DTYPE, "dtype"),
    (dict(norm_weight=FAKE, grad_projections=FAKE), ARG, "exclude"),
])
def test_mixer_backward_rejects(L, change, code, words):
    assert L.sparc_mixer_backward(ctypes.byref(_mixer_bwd(**change)), None) == code
    assert words in _msg(L.sparc_last_error)


def test_null_args_and_status_pointers(L):
    for fn in (L.sparc_mixer_forward, L.sparc_mixer_forward_noalloc, L.sparc_mixer_backward, L.sparc_decode_step,
               L.sparc_real_scan_forward, L.sparc_real_scan_backward):
        assert fn(None, None) == ARG
        assert _msg(L.sparc_last_error) == "null args"
    assert L.sparc_read_status(None, ctypes.byref(ctypes.c_uint()), None) == ARG
    assert L.sparc_read_status(FAKE, None, None) == ARG
    assert L.sparc_clear_status(None, None) == ARG
    assert _msg(L.sparc_last_error) == "null pointer"


def _decode(**kw):
    a = _lib.DecodeArgs(*[FAKE + 16 * i for i in range(13)], 2, 8, _lib.DTYPE_F32)
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("change,code,words", [
    (dict(x=None), ARG, "null tensor"),
    (dict(write_radial_response=None), ARG, "null tensor"),
    (dict(batch=0), SHAPE, "positive"),
    (dict(width=7), SHAPE, "even"),
    (dict(width=4098), SHAPE, "limit"),
    (dict(new_state_r=FAKE + 32), ARG, "alias"),  # new_state_r == state_r
    (dict(dtype=3), DTYPE, "dtype"),
])
def test_decode_rejects(L, change, code, words):
    assert L.sparc_decode_step(ctypes.byref(_decode(**change)), None) == code
    assert words in _msg(L.sparc_last_error)


@pytest.mark.parametrize("change,code,words", [
    (dict(a=None), ARG, "null tensor"),
    (dict(carry=None), ARG, "null tensor"),
    (dict(batch=0), SHAPE, "positive"),
    (dict(channels=-3), SHAPE, "positive"),
    (dict(dtype=2), DTYPE, "dtype"),
    (dict(a_dtype=5), DTYPE, "dtype"),
])
def test_real_scan_rejects(L, change, code, words):
    f = _lib.RealFwdArgs(FAKE, FAKE, FAKE, None, FAKE, FAKE, 1 << 30, 2, 32, 3, _lib.DTYPE_F32, _lib.DTYPE_F32,
                         0, 0, 0)
    for k, v in change.items():
        setattr(f, k, v)
    assert L.sparc_real_scan_forward(ctypes.byref(f), None) == code
    assert words in _msg(L.sparc_last_error)
    bwd = {"a": "grad_a"}.get(next(iter(change)), next(iter(change)))
    r = _lib.RealBwdArgs(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 1 << 30, 2, 32, 3, _lib.DTYPE_F32,
                         _lib.DTYPE_F32, 0)
    setattr(r, bwd, change[next(iter(change))])
    assert L.sparc_real_scan_backward(ctypes.byref(r), None) == code
    assert words in _msg(L.sparc_last_error)


def test_workspace_queries_return_zero_for_invalid_shapes(L):
    assert L.sparc_mixer_workspace_bytes(0, 16, 8, _lib.DTYPE_F32) == 0
    assert L.sparc_mixer_workspace_bytes(2, 16, 7, _lib.DTYPE_F32) == 0
    assert L.sparc_mixer_workspace_bytes(2, 16, 8, 9) == 0
    assert L.sparc_real_workspace_bytes(2, 0, 8, _lib.DTYPE_F32) == 0
    assert L.sparc_real_workspace_bytes(2, 8, 8, 9) == 0
    assert L.sparc_exchange_buffer_bytes(0) == 0 and L.sparc_exchange_buffer_bytes(9) == 0
    assert L.sparc_exchange_buffer_bytes(8) > L.sparc_exchange_buffer_bytes(2) > 0
    assert L.sparc_peer_buffer_bytes(9, 100) == 0 and L.sparc_peer_buffer_bytes(2, 0) == 0
    assert L.sparc_peer_buffer_bytes(2, 100) > 0
    assert L.sparc_mixer_mask_words(0) == 0 and L.sparc_mixer_mask_words(5) == 0


def _rtrl_step(**kw):
    tr = (ctypes.c_void_p * 9)(*[FAKE] * 9)
    ntr = (ctypes.c_void_p * 9)(*[FAKE + 16] * 9)
    a = _lib.RtrlStepArgs(*[FAKE] * 3, None, *[FAKE] * 7, tr, ntr, FAKE, 2, 6, 4, 0)
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_rtrl_rejects(L):
    cases = [(dict(batch=0), SHAPE, "positive"), (dict(batch=70000), SHAPE, "65535"), (dict(modes=0), SHAPE, "positive"),
             (dict(x=None), ARG, "null tensor"), (dict(saved=None), ARG, "null tensor")]
    for change, code, words in cases:
        assert L.sparc_rtrl_step(ctypes.byref(_rtrl_step(**change)), None) == code
        assert words in _msg(L.sparc_rtrl_last_error)
    a = _rtrl_step()
    a.traces[4] = None
    assert L.sparc_rtrl_step(ctypes.byref(a), None) == ARG
    assert "trace" in _msg(L.sparc_rtrl_last_error)
    assert L.sparc_rtrl_step(None, None) == ARG

    def grad(**kw):
        g = _lib.RtrlGradArgs(FAKE, (ctypes.c_void_p * 9)(*[FAKE] * 9), FAKE, (ctypes.c_void_p * 9)(*[FAKE] * 9),
                              FAKE, FAKE, 2, 6, 4)
        for k, v in kw.items():
            setattr(g, k, v)
        return g

    for change, code in ((dict(batch=-1), SHAPE), (dict(input_size=0), SHAPE), (dict(grad_state=None), ARG),
                         (dict(grad_projections=None), ARG)):
        assert L.sparc_rtrl_grad(ctypes.byref(grad(**change)), None) == code
    g = grad()
    g.grad_params[8] = None
    assert L.sparc_rtrl_grad(ctypes.byref(g), None) == ARG
    assert L.sparc_rtrl_grad(None, None) == ARG


def test_gemm_rejects(L):
    def args(**kw):
        a = _lib.ProjGemmArgs(FAKE, FAKE + 4096, FAKE + 8192, None, None, None, None, None, FAKE + 12288, 130, 70,
                              24, 1, 0)
        for k, v in kw.items():
            setattr(a, k, v)
        return a

    cases = [(dict(a=None), ARG, "null"), (dict(status=None), ARG, "null"), (dict(rows=0), SHAPE, "positive"),
             (dict(k=12), SHAPE, "multiple of 8"), (dict(x=FAKE), ARG, "together"),
             (dict(dp=FAKE, c0=FAKE), ARG, "together"), (dict(a=FAKE + 8), ARG, "16-byte aligned"),
             (dict(b=FAKE + 4100), ARG, "16-byte aligned")]
    for change, code, words in cases:
        assert L.sparc_proj_gemm(ctypes.byref(args(**change)), None) == code, change
        assert words in _msg(L.sparc_proj_gemm_last_error), change
    assert L.sparc_proj_gemm(None, None) == ARG


def test_peer_allreduce_rejects(L):
    def args(world=2, rank=0, nseg=2, counts=(3, 5), total=8, status=FAKE, buffers=(FAKE, FAKE + 16)):
        a = _lib.PeerAllreduceArgs()
        for i, c in enumerate(counts):
            a.segments[i] = FAKE + 64 * (i + 1)
            a.counts[i] = c
        a.nseg, a.total, a.world, a.rank, a.scale, a.status = nseg, total, world, rank, 1.0, status
        for r, b in enumerate(buffers):
            a.buffers[r] = b
        return a

    cases = [(dict(world=9), "world"), (dict(world=0), "world"), (dict(rank=2), "rank"), (dict(rank=-1), "rank"),
             (dict(nseg=0), "segments"), (dict(nseg=65), "segments"), (dict(status=None), "status"),
             (dict(counts=(3, 0)), "segment"), (dict(total=9), "add up"), (dict(buffers=(FAKE, None)), "peer buffer")]
    for change, words in cases:
        assert L.sparc_peer_allreduce(ctypes.byref(args(**change)), None) == ARG, change
        assert words in _msg(L.sparc_peer_last_error), change
    assert L.sparc_peer_allreduce(None, None) == ARG
    handle = ctypes.create_string_buffer(64)
    p = ctypes.c_void_p()
    assert L.sparc_peer_buffer_alloc(0, ctypes.byref(p), handle) == ARG
    assert L.sparc_peer_buffer_alloc(1024, None, handle) == ARG
    assert L.sparc_peer_buffer_open(None, ctypes.byref(p)) == ARG
    assert L.sparc_peer_buffer_open(handle, None) == ARG
