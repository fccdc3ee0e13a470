"""The forward entry point that allocates nothing (sparc_mixer_forward_noalloc).

Some callers cannot allocate device memory, e.g. a plugin bound through an FFI into a process
whose memory pool already owns the GPU, or a serving loop that must not call cudaMalloc after
start-up. For them the library keeps the forward's scratch in a fixed 32 MiB array of its own.
These tests call that entry point through the C ABI (ctypes, no workspace passed) several times
in a row, in float32 and bfloat16 and in the plain, block (RMSNorm + residual) and projection
modes, with shapes that shrink and then grow again so that every call finds the previous call's
leftovers in the shared array. Each result is checked against the regular sparc_mixer_forward
within the forward tolerance used elsewhere (1e-4 relative l2 for float32, 2e-2 for bfloat16),
and the array's status word, read and cleared through the entry points made for it, must stay 0.
A problem too large for the array is refused with a clear error, and the size query agrees with
the refusal. The file is collected last on purpose: if it fails, a run that stops at the first
failure has already run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

NAMES = ("nu_log", "theta_log", "phase_direction", "radial_direction", "write_log_gain",
         "write_phase_response", "write_radial_response")
TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


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
    return {n: getattr(m, n).detach().float().cuda().contiguous() for n in NAMES}


def _inputs(mode, B, T, W, dtype, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(B, T, W, generator=gen, device="cuda").to(dtype)
    extra = {}
    if mode == "block":
        extra["norm_weight"] = (1.0 + 0.1 * torch.randn(W, generator=gen, device="cuda")).contiguous()
    if mode == "proj":
        extra["projections"] = (0.5 * torch.randn(B, T, 2, generator=gen, device="cuda")).contiguous()
    return x, extra


def _call(entry, x, params, extra, workspace=None):
    from sparc_b200 import _lib

    L = _lib.lib()
    B, T, W = x.shape
    M = W // 2
    dt = _lib.dtype_code(x.dtype)
    y = torch.empty_like(x)
    carry = torch.empty((B, L.sparc_mixer_carry_chunks(T, dt), M, 2), device=x.device)
    last_r = torch.empty((B, M), device=x.device)
    last_i = torch.empty((B, M), device=x.device)
    controls = torch.empty((B, T, L.sparc_mixer_controls_floats()), device=x.device)
    nw = extra.get("norm_weight")
    mask = (torch.empty((B, T, L.sparc_mixer_mask_words(W)), dtype=torch.int32, device=x.device)
            if nw is not None else None)
    proj = extra.get("projections")
    p = params
    if proj is not None:  # projection mode: no direction vectors
        plist = [p["nu_log"], p["theta_log"], None, None, p["write_log_gain"], p["write_phase_response"],
                 p["write_radial_response"]]
    else:
        plist = [p[n] for n in NAMES]
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (workspace.data_ptr(), workspace.numel())
    a = _lib.MixerFwdArgs(x.data_ptr(), y.data_ptr(), *[_lib.ptr(t) for t in plist], None, None,
                          last_r.data_ptr(), last_i.data_ptr(), carry.data_ptr(), controls.data_ptr(), None,
                          _lib.ptr(nw), 1e-6, _lib.ptr(mask), _lib.ptr(proj), 0, ws_ptr, ws_bytes,
                          B, T, W, dt, 0)
    rc = getattr(L, entry)(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    return rc, (y, last_r, last_i, carry)


def _rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm()).item()


def _status():
    from sparc_b200 import _lib

    st = ctypes.c_uint(7)
    rc = _lib.lib().sparc_mixer_noalloc_read_status(ctypes.byref(st), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.lib().sparc_last_error()
    return st.value


# shrink, then grow past the first size: each call finds the previous call's scratch contents
SHAPES = [(4, 1000, 256), (2, 333, 64), (3, 1500, 600)]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("mode", ["plain", "block", "proj"])
def test_noalloc_forward_matches_regular_forward_in_a_row(mode, dtype):
    from sparc_b200 import _lib

    L = _lib.lib()
    assert L.sparc_mixer_noalloc_scratch_bytes() == 32 << 20
    stream = torch.cuda.current_stream().cuda_stream
    assert L.sparc_mixer_noalloc_clear_status(stream) == 0
    for call, (B, T, W) in enumerate(SHAPES):
        seed = 10 * call + 1
        params = _params(W, seed)
        x, extra = _inputs(mode, B, T, W, dtype, seed)
        dt = _lib.dtype_code(dtype)
        assert 0 < L.sparc_mixer_noalloc_scratch_needed(B, T, W, dt) <= L.sparc_mixer_noalloc_scratch_bytes()
        ws = torch.zeros(L.sparc_mixer_workspace_bytes(B, T, W, dt), dtype=torch.uint8, device="cuda")
        rc0, ref = _call("sparc_mixer_forward", x, params, extra, ws)
        rc1, got = _call("sparc_mixer_forward_noalloc", x, params, extra)
        torch.cuda.synchronize()
        assert rc0 == 0 and rc1 == 0, (call, rc0, rc1, L.sparc_last_error())
        for name, g, r in zip(("y", "last_r", "last_i", "carry"), got, ref):
            assert _rel(g, r) < TOL[dtype], (mode, call, name, _rel(g, r))
        assert _status() == 0, (mode, call)


def test_noalloc_rejects_problems_above_its_scratch():
    from sparc_b200 import _lib

    L = _lib.lib()
    B, T, W = 64, 1024, 2048
    need = L.sparc_mixer_noalloc_scratch_needed(B, T, W, _lib.DTYPE_F32)
    assert need > L.sparc_mixer_noalloc_scratch_bytes()
    params = _params(W, 3)
    x = torch.zeros(B, T, W, device="cuda")
    rc, _ = _call("sparc_mixer_forward_noalloc", x, params, {})
    assert rc == -4
    assert b"built-in" in L.sparc_last_error()
    assert _status() == 0
