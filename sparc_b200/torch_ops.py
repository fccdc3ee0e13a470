"""PyTorch operators over the libsparc_b200 C ABI: ``torch.ops.sparc_b200.mixer_forward``,
``mixer_backward``, ``decode_step``, ``real_scan_forward`` and ``real_scan_backward``
(registered by csrc_torch/torch_ops.cpp with TORCH_LIBRARY, CUDA dispatch key). They take and
return CUDA tensors and run on PyTorch's current stream; `load()` makes them available."""
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
    return torch.ops.sparc_b200
