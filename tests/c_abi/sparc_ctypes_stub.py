"""ctypes stub a maintainer would add to the reference (Botwwt/sparc, sparc-kernal) to route
SPARCMixer.forward (sparc.py:90-91 -> run_sequence, forward/scan.py:1398) through
libsparc_b200.so. The library path comes from SPARC_B200_LIBRARY, else the loader's search
path. tests/test_capi.py loads this file and checks its struct layout against the header."""
import ctypes
import os

import torch

lib = ctypes.CDLL(os.environ.get("SPARC_B200_LIBRARY", "libsparc_b200.so"))
lib.sparc_last_error.restype = ctypes.c_char_p          # pointers and 64-bit sizes need their
lib.sparc_mixer_workspace_bytes.restype = ctypes.c_size_t  # return types declared (ctypes
lib.sparc_mixer_workspace_bytes.argtypes = [ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int, ctypes.c_int]
lib.sparc_mixer_carry_chunks.restype = ctypes.c_longlong   # defaults to a 32-bit int)
lib.sparc_mixer_carry_chunks.argtypes = [ctypes.c_longlong, ctypes.c_int]

class SparcMixerFwdArgs(ctypes.Structure):   # field order of include/sparc_b200.h
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "x", "y", "nu_log", "theta_log", "phase_direction", "radial_direction",
        "write_log_gain", "write_phase_response", "write_radial_response",
        "h0_r", "h0_i", "last_r", "last_i", "carry", "controls", "reset")] + [
        ("norm_weight", ctypes.c_void_p), ("norm_eps", ctypes.c_float), ("relu_mask", ctypes.c_void_p),
        ("projections", ctypes.c_void_p), ("content_linear", ctypes.c_int),
        ("workspace", ctypes.c_void_p)] + [
        ("workspace_bytes", ctypes.c_size_t), ("batch", ctypes.c_longlong),
        ("length", ctypes.c_longlong), ("width", ctypes.c_int), ("dtype", ctypes.c_int),
        ("max_spin", ctypes.c_uint), ("y_im", ctypes.c_void_p), ("states", ctypes.c_void_p)]

def run_sequence(module, x, return_cache=False):
    B, T, W = x.shape
    dt = 1 if x.dtype == torch.bfloat16 else 0
    y = torch.empty_like(x)
    carry = torch.empty(B, lib.sparc_mixer_carry_chunks(T, dt), W // 2, 2, device=x.device)
    controls = torch.empty(B, T, lib.sparc_mixer_controls_floats(), device=x.device)  # saved, like carry
    last = [torch.empty(B, W // 2, device=x.device) for _ in range(2)]
    ws = torch.zeros(lib.sparc_mixer_workspace_bytes(B, T, W, dt), dtype=torch.uint8, device=x.device)
    p = [getattr(module, n).detach().float().contiguous() for n in (
        "nu_log", "theta_log", "phase_direction", "radial_direction",
        "write_log_gain", "write_phase_response", "write_radial_response")]
    a = SparcMixerFwdArgs(x.data_ptr(), y.data_ptr(), *[t.data_ptr() for t in p], None, None,
                          last[0].data_ptr(), last[1].data_ptr(), carry.data_ptr(), controls.data_ptr(),
                          None, None, 0.0, None, None, 0, ws.data_ptr(), ws.numel(), B, T, W, dt, 0)
    rc = lib.sparc_mixer_forward(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    if rc:
        raise RuntimeError(f"sparc_mixer_forward: {rc}: {lib.sparc_last_error().decode()}")
    return y, ((last[0], last[1]) if return_cache else None)
