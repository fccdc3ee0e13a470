"""A plain-C host program drives the mixer through the C ABI alone (tests/c_abi/mixer_from_c.c,
compiled here with gcc against include/sparc_b200.h and libsparc_b200.so); its outputs match the
float64 oracle at the float32 tolerances."""
import os
import subprocess

import numpy as np
import pytest

from oracle import sparc_oracle as O

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
B, T, W = 2, 37, 10
M = W // 2


def _inputs():
    i = np.arange(B * T * W, dtype=np.float32)
    x = (np.sin(np.float32(0.37) * i) * np.float32(1.3)).astype(np.float32).reshape(B, T, W)
    dy = np.cos(np.float32(0.21) * i + np.float32(0.5)).astype(np.float32).reshape(B, T, W)
    m = np.arange(M, dtype=np.float32)
    j = np.arange(W + 1, dtype=np.float32)
    p = {"nu_log": -3.0 + 0.4 * m, "theta_log": -1.0 + 0.3 * m, "write_log_gain": -0.5 - 0.1 * m,
         "write_phase_response": 0.3 * np.sin(m), "write_radial_response": 0.2 * np.cos(m),
         "phase_direction": 0.15 * np.sin(1.7 * j), "radial_direction": 0.15 * np.cos(1.3 * j),
         "energy_response": np.zeros(M)}
    return x, dy, {k: np.asarray(v, np.float32).astype(np.float64) for k, v in p.items()}


def test_c_program_matches_oracle(tmp_path):
    from sparc_b200 import _build

    lib = _build.build()
    exe = tmp_path / "mixer_from_c"
    cmd = ["gcc", "-O2", "-o", str(exe), os.path.join(ROOT, "tests", "c_abi", "mixer_from_c.c"),
           "-I", os.path.join(ROOT, "include"), "-I", "/usr/local/cuda/include",
           "-L", os.path.dirname(lib), "-lsparc_b200", "-L", "/usr/local/cuda/lib64", "-lcudart", "-lm",
           f"-Wl,-rpath,{os.path.dirname(lib)}", "-Wl,-rpath,/usr/local/cuda/lib64"]
    subprocess.run(cmd, check=True)
    out = tmp_path / "out.bin"
    r = subprocess.run([str(exe), str(out)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    v = np.fromfile(out, dtype=np.float32)
    n = B * T * W
    y, dx = v[:n].reshape(B, T, W), v[n:2 * n].reshape(B, T, W)
    sizes = [M, M, W + 1, W + 1, M, M, M, M]
    names = ["nu_log", "theta_log", "phase_direction", "radial_direction", "write_log_gain", "energy_response",
             "write_phase_response", "write_radial_response"]
    grads, off = {}, 2 * n
    for k, s in zip(names, sizes):
        grads[k] = v[off:off + s]
        off += s
    x, dy, p = _inputs()
    P = O.Params.from_mapping(p)
    y_ref, _, _ = O.sparc_forward(x.astype(np.float64), P)
    g_ref = O.sparc_backward(x.astype(np.float64), P, dy.astype(np.float64))
    assert O.rel_l2(y, y_ref) < 1e-4
    assert O.rel_l2(dx, g_ref["x"]) < 1e-3
    for k in names:
        if k != "energy_response":
            assert O.rel_l2(grads[k], g_ref[k]) < 1e-3, k
    assert np.all(grads["energy_response"] == 0)
