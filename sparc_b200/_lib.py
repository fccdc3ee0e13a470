"""ctypes binding of libsparc_b200.so (the C ABI declared in include/sparc_b200.h).

This is the only place Python touches the library. Tensors cross the boundary as raw device
pointers (``tensor.data_ptr()``) and the current CUDA stream as a ``cudaStream_t`` handle.
There is no fallback: if the library or a CUDA device is missing, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
# SPARC_B200_LIBRARY selects another build of the library (for example to compare two builds)
LIB_PATH = os.environ.get("SPARC_B200_LIBRARY") or os.path.join(_PKG, "libsparc_b200.so")

OK = 0
ERR_NAMES = {-1: "bad argument", -2: "bad shape", -3: "bad dtype", -4: "workspace", -5: "launch"}
DTYPE_F32 = 0
DTYPE_BF16 = 1
STATUS_TIMEOUT = 1

_vp = ctypes.c_void_p
_ll = ctypes.c_longlong


class MixerFwdArgs(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("y", _vp),
        ("nu_log", _vp), ("theta_log", _vp), ("phase_direction", _vp), ("radial_direction", _vp),
        ("write_log_gain", _vp), ("write_phase_response", _vp), ("write_radial_response", _vp),
        ("h0_r", _vp), ("h0_i", _vp), ("last_r", _vp), ("last_i", _vp), ("carry", _vp),
        ("controls", _vp), ("reset", _vp),
        ("norm_weight", _vp), ("norm_eps", ctypes.c_float), ("relu_mask", _vp),
        ("projections", _vp), ("content_linear", ctypes.c_int),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
        ("batch", _ll), ("length", _ll), ("width", ctypes.c_int), ("dtype", ctypes.c_int),
        ("max_spin", ctypes.c_uint), ("y_im", _vp), ("states", _vp),
    ]


class MixerBwdArgs(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("y", _vp), ("dy", _vp), ("dx", _vp),
        ("nu_log", _vp), ("theta_log", _vp), ("phase_direction", _vp), ("radial_direction", _vp),
        ("write_log_gain", _vp), ("write_phase_response", _vp), ("write_radial_response", _vp),
        ("h0_r", _vp), ("h0_i", _vp), ("grad_last_r", _vp), ("grad_last_i", _vp),
        ("grad_h0_r", _vp), ("grad_h0_i", _vp), ("carry", _vp), ("controls", _vp),
        ("norm_weight", _vp), ("relu_mask", _vp), ("grad_norm_weight", _vp),
        ("grad_nu_log", _vp), ("grad_theta_log", _vp), ("grad_phase_direction", _vp),
        ("grad_radial_direction", _vp), ("grad_write_log_gain", _vp), ("grad_energy_response", _vp),
        ("grad_write_phase_response", _vp), ("grad_write_radial_response", _vp),
        ("grad_projections", _vp), ("content_linear", ctypes.c_int),
        ("exchange_buffers", _vp * 8), ("exchange_world", ctypes.c_int), ("exchange_rank", ctypes.c_int),
        ("exchange_status", _vp),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
        ("batch", _ll), ("length", _ll), ("width", ctypes.c_int), ("dtype", ctypes.c_int),
        ("max_spin", ctypes.c_uint), ("states", _vp),
    ]


class DecodeArgs(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("y", _vp), ("state_r", _vp), ("state_i", _vp),
        ("new_state_r", _vp), ("new_state_i", _vp),
        ("nu_log", _vp), ("theta_log", _vp), ("phase_direction", _vp), ("radial_direction", _vp),
        ("write_log_gain", _vp), ("write_phase_response", _vp), ("write_radial_response", _vp),
        ("batch", _ll), ("width", ctypes.c_int), ("dtype", ctypes.c_int),
    ]


class RealFwdArgs(ctypes.Structure):
    _fields_ = [
        ("a", _vp), ("b", _vp), ("out", _vp), ("last", _vp), ("carry", _vp),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
        ("batch", _ll), ("length", _ll), ("channels", _ll), ("dtype", ctypes.c_int), ("a_dtype", ctypes.c_int),
        ("max_spin", ctypes.c_uint),
        ("inject_enable", ctypes.c_int), ("inject_tile", _ll),
    ]


class RealBwdArgs(ctypes.Structure):
    _fields_ = [
        ("a", _vp), ("b", _vp), ("grad_out", _vp), ("carry", _vp), ("grad_a", _vp), ("grad_b", _vp),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
        ("batch", _ll), ("length", _ll), ("channels", _ll), ("dtype", ctypes.c_int), ("a_dtype", ctypes.c_int),
        ("max_spin", ctypes.c_uint),
    ]


class ComplexFwdArgs(ctypes.Structure):
    _fields_ = [
        ("ar", _vp), ("ai", _vp), ("br", _vp), ("bi", _vp), ("out_r", _vp), ("out_i", _vp),
        ("last_r", _vp), ("last_i", _vp), ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
        ("batch", _ll), ("length", _ll), ("modes", _ll), ("a_dtype", ctypes.c_int), ("b_dtype", ctypes.c_int),
    ]


class ComplexBwdArgs(ctypes.Structure):
    _fields_ = [
        ("ar", _vp), ("ai", _vp), ("out_r", _vp), ("out_i", _vp), ("grad_out_r", _vp), ("grad_out_i", _vp),
        ("grad_ar", _vp), ("grad_ai", _vp), ("grad_br", _vp), ("grad_bi", _vp),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
        ("batch", _ll), ("length", _ll), ("modes", _ll), ("a_dtype", ctypes.c_int), ("b_dtype", ctypes.c_int),
    ]


class RtrlStepArgs(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("content", _vp), ("projections", _vp), ("reset", _vp), ("state", _vp), ("new_state", _vp),
        ("decay_log", _vp), ("frequency_log", _vp), ("write_log_gain", _vp), ("write_phase_response", _vp),
        ("write_retention_response", _vp), ("traces", _vp * 9), ("new_traces", _vp * 9), ("saved", _vp),
        ("batch", _ll), ("input_size", ctypes.c_int), ("modes", ctypes.c_int), ("content_linear", ctypes.c_int),
    ]


class RtrlGradArgs(ctypes.Structure):
    _fields_ = [
        ("grad_state", _vp), ("traces", _vp * 9), ("saved", _vp), ("grad_params", _vp * 9),
        ("grad_content", _vp), ("grad_projections", _vp),
        ("batch", _ll), ("input_size", ctypes.c_int), ("modes", ctypes.c_int),
    ]


class ProjGemmArgs(ctypes.Structure):
    _fields_ = [
        ("a", _vp), ("b", _vp), ("out", _vp), ("x", _vp), ("skip", _vp), ("dp", _vp), ("c0", _vp), ("c1", _vp),
        ("status", _vp), ("rows", _ll), ("n", ctypes.c_int), ("k", ctypes.c_int), ("out_f32", ctypes.c_int),
        ("max_spin", ctypes.c_uint), ("a_mn", ctypes.c_int), ("b_mn", ctypes.c_int),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
    ]


class ProjRowdotArgs(ctypes.Structure):
    _fields_ = [("x", _vp), ("c", _vp), ("p", _vp), ("rows", _ll), ("w", ctypes.c_int), ("dtype", ctypes.c_int)]


class ProjColsumArgs(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("dp", _vp), ("dy", _vp), ("d_ctl", _vp), ("d_skip", _vp), ("workspace", _vp),
        ("workspace_bytes", ctypes.c_size_t), ("rows", _ll), ("w", ctypes.c_int), ("dtype", ctypes.c_int),
    ]


class PeerAllreduceArgs(ctypes.Structure):
    _fields_ = [
        ("segments", _vp * 64), ("counts", _ll * 64), ("nseg", ctypes.c_int), ("total", _ll),
        ("buffers", _vp * 8), ("world", ctypes.c_int), ("rank", ctypes.c_int), ("scale", ctypes.c_float),
        ("max_spin", ctypes.c_uint), ("status", _vp), ("inject_skip_publish", ctypes.c_int),
    ]


# every symbol declared in include/sparc_b200.h, with its ctypes signature
SIGNATURES = {
    "sparc_last_error": (ctypes.c_char_p, []),
    "sparc_mixer_chunk_tokens": (_ll, [ctypes.c_int]),
    "sparc_mixer_carry_chunks": (_ll, [_ll, ctypes.c_int]),
    "sparc_mixer_mask_words": (ctypes.c_int, [ctypes.c_int]),
    "sparc_mixer_controls_floats": (ctypes.c_int, []),
    "sparc_mixer_workspace_bytes": (ctypes.c_size_t, [_ll, _ll, ctypes.c_int, ctypes.c_int]),
    "sparc_mixer_forward": (ctypes.c_int, [ctypes.POINTER(MixerFwdArgs), _vp]),
    "sparc_mixer_backward": (ctypes.c_int, [ctypes.POINTER(MixerBwdArgs), _vp]),
    "sparc_mixer_noalloc_scratch_bytes": (ctypes.c_size_t, []),
    "sparc_mixer_noalloc_scratch_needed": (ctypes.c_size_t, [_ll, _ll, ctypes.c_int, ctypes.c_int]),
    "sparc_mixer_forward_noalloc": (ctypes.c_int, [ctypes.POINTER(MixerFwdArgs), _vp]),
    "sparc_mixer_noalloc_read_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint), _vp]),
    "sparc_mixer_noalloc_clear_status": (ctypes.c_int, [_vp]),
    "sparc_decode_step": (ctypes.c_int, [ctypes.POINTER(DecodeArgs), _vp]),
    "sparc_real_chunk_tokens": (_ll, []),
    "sparc_real_carry_chunks": (_ll, [_ll]),
    "sparc_real_workspace_bytes": (ctypes.c_size_t, [_ll, _ll, _ll, ctypes.c_int]),
    "sparc_real_scan_forward": (ctypes.c_int, [ctypes.POINTER(RealFwdArgs), _vp]),
    "sparc_real_scan_backward": (ctypes.c_int, [ctypes.POINTER(RealBwdArgs), _vp]),
    "sparc_complex_chunk_tokens": (_ll, []),
    "sparc_complex_workspace_bytes": (ctypes.c_size_t, [_ll, _ll, _ll]),
    "sparc_complex_scan_forward": (ctypes.c_int, [ctypes.POINTER(ComplexFwdArgs), _vp]),
    "sparc_complex_scan_backward": (ctypes.c_int, [ctypes.POINTER(ComplexBwdArgs), _vp]),
    "sparc_read_status": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_uint), _vp]),
    "sparc_clear_status": (ctypes.c_int, [_vp, _vp]),
    "sparc_rtrl_saved_floats": (ctypes.c_int, []),
    "sparc_rtrl_step": (ctypes.c_int, [ctypes.POINTER(RtrlStepArgs), _vp]),
    "sparc_rtrl_grad": (ctypes.c_int, [ctypes.POINTER(RtrlGradArgs), _vp]),
    "sparc_rtrl_last_error": (ctypes.c_char_p, []),
    "sparc_proj_gemm": (ctypes.c_int, [ctypes.POINTER(ProjGemmArgs), _vp]),
    "sparc_proj_gemm_last_error": (ctypes.c_char_p, []),
    "sparc_proj_colsum_workspace_bytes": (ctypes.c_size_t, [_ll, ctypes.c_int]),
    "sparc_proj_gemm_workspace_bytes": (ctypes.c_size_t, [_ll, ctypes.c_int, ctypes.c_int]),
    "sparc_proj_colsum": (ctypes.c_int, [ctypes.POINTER(ProjColsumArgs), _vp]),
    "sparc_proj_rowdot": (ctypes.c_int, [ctypes.POINTER(ProjRowdotArgs), _vp]),
    "sparc_exchange_buffer_bytes": (ctypes.c_size_t, [ctypes.c_int]),
    "sparc_peer_buffer_bytes": (ctypes.c_size_t, [ctypes.c_int, _ll]),
    "sparc_peer_buffer_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(_vp), _vp]),
    "sparc_peer_buffer_open": (ctypes.c_int, [_vp, ctypes.POINTER(_vp)]),
    "sparc_peer_buffer_close": (ctypes.c_int, [_vp]),
    "sparc_peer_buffer_free": (ctypes.c_int, [_vp]),
    "sparc_peer_allreduce": (ctypes.c_int, [ctypes.POINTER(PeerAllreduceArgs), _vp]),
    "sparc_peer_last_error": (ctypes.c_char_p, []),
    "sparc_timing_enable": (ctypes.c_int, [ctypes.c_int]),
    "sparc_timing_kernel_name": (ctypes.c_char_p, [ctypes.c_int]),
    "sparc_timing_read": (ctypes.c_int, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_longlong),
                                         ctypes.c_int]),
}

_lib = None
_lock = threading.Lock()


def load_library(path: str = LIB_PATH):
    """Load (once) and return the CDLL. Raises if the library is missing."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise RuntimeError(
                    f"{path} is missing: build it with `python -m sparc_b200._build` "
                    "(there is no CPU or Python fallback for the SPARC kernels)")
            lib = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def lib():
    return load_library()


def check(rc: int, what: str):
    if rc != OK:
        msg = lib().sparc_last_error()
        msg = msg.decode() if msg else ""
        raise RuntimeError(f"{what} failed ({ERR_NAMES.get(rc, rc)}): {msg}")


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return DTYPE_F32
    if dtype == torch.bfloat16:
        return DTYPE_BF16
    raise TypeError(f"sparc_b200 supports float32 and bfloat16 activations, got {dtype}")


def require_cuda(t: torch.Tensor, name: str):
    if not t.is_cuda:
        raise RuntimeError(f"sparc_b200: {name} must be a CUDA tensor (there is no CPU path)")




def ptr(t):
    return None if t is None else t.data_ptr()


def stream_handle(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class _Workspaces:
    """Zero-initialised scratch per (device, stream), grown on demand.

    The library keeps its launch counters and lookback flags in the workspace, so one is
    reused across launches on a stream; concurrent streams get their own."""

    def __init__(self):
        self._ws = {}

    def get(self, device: torch.device, nbytes: int, kind: str = "mixer") -> torch.Tensor:
        """`kind` keeps the real-mode scan's status words apart from the mixer's scratch: a
        scan recognises the words of its own earlier launches by their epoch, not arbitrary
        data another family of kernels left behind."""
        key = (device.index, torch.cuda.current_stream(device).cuda_stream, kind)
        ws = self._ws.get(key)
        if ws is None or ws.numel() < nbytes:
            size = max(nbytes, 1 << 20)
            if ws is not None:
                size = max(size, int(ws.numel() * 1.25))
            ws = torch.zeros(size, dtype=torch.uint8, device=device)
            self._ws[key] = ws
        return ws

    def all(self, kinds=("mixer", "real")):
        """The cached workspaces of the given kinds: by default those that begin with the
        library's launch state and status word (the "gemm" and "complex" kinds hold scratch
        values from their first byte)."""
        return [ws for (_, _, kind), ws in self._ws.items() if kind in kinds]


WORKSPACES = _Workspaces()


def read_status(ws: torch.Tensor) -> int:
    st = ctypes.c_uint(0)
    check(lib().sparc_read_status(ws.data_ptr(), ctypes.byref(st), stream_handle(ws.device)),
          "sparc_read_status")
    return int(st.value)


def clear_status(ws: torch.Tensor):
    check(lib().sparc_clear_status(ws.data_ptr(), stream_handle(ws.device)), "sparc_clear_status")


def kernel_times(reset_only: bool = False):
    """Per-kernel device time recorded since the last call while timing was enabled
    (sparc_timing_enable): {kernel name: (total ms, launches)} for kernels that ran."""
    L = lib()
    n = 32
    ms = (ctypes.c_double * n)()
    cnt = (ctypes.c_longlong * n)()
    k = L.sparc_timing_read(ms, cnt, n)
    if reset_only:
        return {}
    return {L.sparc_timing_kernel_name(i).decode(): (ms[i], cnt[i]) for i in range(k) if cnt[i] > 0}
