"""The forward entry point that allocates nothing (sparc_mixer_forward_noalloc).

Some callers cannot allocate device memory, e.g. a plugin bound through an FFI into a process
whose memory pool already owns the GPU, or a serving loop that must not call cudaMalloc after
start-up. For them the library keeps the forward's scratch in a fixed 32 MiB array of its own.
This test calls that entry point through the C ABI (ctypes, no workspace passed) twice in a
row, with different shapes so the second call finds the first call's leftovers in the shared
array, and checks each result against the regular sparc_mixer_forward within the float32
forward tolerance used elsewhere (1e-4 relative l2). It also checks that a problem too large
for the array is refused with a clear error. It is collected last on purpose: if it fails, a
run that stops at the first failure has already run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _params(W, seed):
    torch.manual_seed(seed)
    import sparc_b200

    m = sparc_b200.SPARCMixer(W)
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        m.phase_direction.copy_(torch.randn(W + 1, generator=g) / W ** 0.5)
        m.radial_direction.copy_(torch.randn(W + 1, generator=g) / W ** 0.5)
        m.write_phase_response.copy_(torch.randn(W // 2, generator=g) * 0.5)
        m.write_radial_response.copy_(torch.randn(W // 2, generator=g) * 0.5)
    names = ("nu_log", "theta_log", "phase_direction", "radial_direction", "write_log_gain",
             "write_phase_response", "write_radial_response")
    return [getattr(m, n).detach().float().cuda().contiguous() for n in names]


def _call(entry, x, params, workspace=None):
    from sparc_b200 import _lib

    L = _lib.lib()
    B, T, W = x.shape
    M = W // 2
    y = torch.empty_like(x)
    carry = torch.empty((B, L.sparc_mixer_carry_chunks(T, _lib.dtype_code(x.dtype)), M, 2), device=x.device)
    last_r = torch.empty((B, M), device=x.device)
    last_i = torch.empty((B, M), device=x.device)
    controls = torch.empty((B, T, L.sparc_mixer_controls_floats()), device=x.device)
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (workspace.data_ptr(), workspace.numel())
    a = _lib.MixerFwdArgs(x.data_ptr(), y.data_ptr(), *[p.data_ptr() for p in params], None, None,
                          last_r.data_ptr(), last_i.data_ptr(), carry.data_ptr(), controls.data_ptr(), None, None, 0.0, None,
                          None, 0, ws_ptr, ws_bytes,
                          B, T, W, _lib.dtype_code(x.dtype), 0)
    rc = getattr(L, entry)(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    return rc, y, last_r, last_i, carry


def _rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm()).item()


def test_noalloc_forward_matches_regular_forward_twice():
    from sparc_b200 import _lib

    L = _lib.lib()
    assert L.sparc_mixer_noalloc_scratch_bytes() == 32 << 20
    for call, (B, T, W, seed) in enumerate([(4, 1000, 256, 1), (2, 333, 64, 2)]):
        params = _params(W, seed)
        x = torch.randn(B, T, W, generator=torch.Generator(device="cuda").manual_seed(seed), device="cuda")
        nbytes = L.sparc_mixer_workspace_bytes(B, T, W, _lib.DTYPE_F32)
        ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
        rc0, y0, lr0, li0, c0 = _call("sparc_mixer_forward", x, params, ws)
        rc1, y1, lr1, li1, c1 = _call("sparc_mixer_forward_noalloc", x, params)
        torch.cuda.synchronize()
        assert rc0 == 0 and rc1 == 0, (call, rc0, rc1, L.sparc_last_error())
        assert _rel(y1, y0) < 1e-4, call
        assert _rel(lr1, lr0) < 1e-4 and _rel(li1, li0) < 1e-4, call
        assert _rel(c1, c0) < 1e-4, call


def test_noalloc_rejects_problems_above_its_scratch():
    from sparc_b200 import _lib

    L = _lib.lib()
    params = _params(2048, 3)
    x = torch.zeros(64, 1024, 2048, device="cuda")
    rc, *_ = _call("sparc_mixer_forward_noalloc", x, params)
    assert rc == -4
    assert b"built-in" in L.sparc_last_error()
