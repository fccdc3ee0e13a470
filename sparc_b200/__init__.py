"""B200-native SPARC hot path: a drop-in for the reference ``sparc-kernal`` PyTorch API.

    from sparc_b200 import SPARCMixer, real_scan, real_chunk_scan, real_scan_with_last
    from sparc_b200 import complex_scan, complex_scan_with_last
    from sparc_b200 import sparc_scan, sparc_chunk_scan, sparc_tiled_serial_scan  # scan level

All compute runs in the sm_100a kernels of ``libsparc_b200.so`` (C ABI in
``include/sparc_b200.h``), loaded through ctypes on first use. There is no CPU path.
"""
from .mixer import (SPARCMixer, prepare_decode, run_decode_step, run_sequence, sparc_block, sparc_decode_step,
                    sparc_eager_step, sparc_mixer)
from .stack import SPARCBlock, SPARCStack
from .projection import SPARCSequenceLayer, sparc_projection_states, sparc_sequence_layer
from .rtrl import SPARCRTRLCell, initialize_carry, initialize_traces, rtrl_step, stored_rtrl_step
from .real import real_chunk_scan, real_scan, real_scan_with_last
from .complex import complex_scan, complex_scan_with_last
from .scan import (sparc_chunk_scan, sparc_scan, sparc_scan_precomputed_decay, sparc_scan_with_last,
                   sparc_tiled_serial_scan, sparc_training_scan_dispatch)
from . import _lib


def library_path() -> str:
    return _lib.LIB_PATH


def check_status(clear: bool = True) -> None:
    """Raise if any kernel launch on a cached workspace recorded a bounded wait that ran out (a
    tile kernel's wait on its TMA copies, or the real scan's lookback). The tensor-core product
    and the multi-GPU exchanges keep their own status words (gemm.gemm_status, the reducers'
    timed_out()).

    Synchronises the streams that own the workspaces."""
    for ws in _lib.WORKSPACES.all():
        st = _lib.read_status(ws)
        if st:
            if clear:
                _lib.clear_status(ws)
            raise RuntimeError(f"sparc_b200: a bounded wait in a kernel timed out (status {st:#x})")


__all__ = ["SPARCMixer", "sparc_mixer", "sparc_block", "SPARCBlock", "SPARCStack", "sparc_decode_step", "sparc_eager_step",
           "SPARCSequenceLayer", "sparc_sequence_layer", "sparc_projection_states",
           "SPARCRTRLCell", "rtrl_step", "stored_rtrl_step", "initialize_carry", "initialize_traces",
           "real_scan", "real_chunk_scan", "real_scan_with_last", "complex_scan", "complex_scan_with_last",
           "sparc_scan", "sparc_chunk_scan",
           "sparc_scan_with_last", "sparc_tiled_serial_scan", "sparc_training_scan_dispatch",
           "sparc_scan_precomputed_decay", "run_sequence", "prepare_decode", "run_decode_step", "check_status",
           "library_path"]
