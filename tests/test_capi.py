"""The C-ABI library loads without a GPU and exports every function include/sparc_b200.h
declares, with the signatures the Python binding uses. No compute call is made here."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "sparc_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(sparc_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from sparc_b200 import _build, _lib

    _build.build()
    return _lib.load_library()


def test_every_declared_symbol_is_exported(lib):
    from sparc_b200 import _lib

    names = _declared()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_struct_layouts_match_header():
    """Field order of the ctypes structures equals the C structs' (parsed from the header)."""
    from sparc_b200 import _lib

    src = open(os.path.join(ROOT, "include", "sparc_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    for cname, py in (("SparcMixerFwdArgs", _lib.MixerFwdArgs), ("SparcMixerBwdArgs", _lib.MixerBwdArgs),
                      ("SparcDecodeArgs", _lib.DecodeArgs), ("SparcRealFwdArgs", _lib.RealFwdArgs),
                      ("SparcRealBwdArgs", _lib.RealBwdArgs), ("SparcRtrlStepArgs", _lib.RtrlStepArgs),
                      ("SparcRtrlGradArgs", _lib.RtrlGradArgs), ("SparcProjGemmArgs", _lib.ProjGemmArgs),
                      ("SparcPeerAllreduceArgs", _lib.PeerAllreduceArgs),
                      ("SparcComplexFwdArgs", _lib.ComplexFwdArgs), ("SparcComplexBwdArgs", _lib.ComplexBwdArgs),
                      ("SparcProjColsumArgs", _lib.ProjColsumArgs), ("SparcProjRowdotArgs", _lib.ProjRowdotArgs)):
        body = re.search(r"typedef struct %s \{(.*?)\}" % cname, src, flags=re.S).group(1)
        fields = re.findall(r"(\w+)\s*(?:\[\w+\])?\s*;", body)
        assert fields == [f[0] for f in py._fields_], cname


def test_host_only_queries(lib):
    from sparc_b200 import _lib

    assert lib.sparc_mixer_chunk_tokens(_lib.DTYPE_BF16) == 16
    assert lib.sparc_mixer_chunk_tokens(_lib.DTYPE_F32) == 8
    assert lib.sparc_mixer_carry_chunks(2048, _lib.DTYPE_BF16) == 128
    assert lib.sparc_mixer_carry_chunks(37, _lib.DTYPE_F32) == 5
    assert lib.sparc_real_carry_chunks(33) == 2 and lib.sparc_real_chunk_tokens() == 32
    assert lib.sparc_complex_chunk_tokens() == 32
    assert lib.sparc_complex_workspace_bytes(2, 33, 5) == 256 + 2 * 2 * 5 * 24
    assert lib.sparc_complex_workspace_bytes(70000, 8, 8) == 0  # beyond the launch grid
    assert lib.sparc_mixer_controls_floats() == 16  # the per-token record the kernels write
    assert lib.sparc_mixer_mask_words(2048) == 64 and lib.sparc_mixer_mask_words(600) == 32
    assert lib.sparc_mixer_mask_words(7) == 0
    assert lib.sparc_rtrl_saved_floats() == 8


def test_no_cpu_fallback():
    import torch

    import sparc_b200

    if torch.cuda.is_available():
        pytest.skip("checks the no-GPU behaviour")
    m = sparc_b200.SPARCMixer(8)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.randn(1, 4, 8))
    with pytest.raises(RuntimeError, match="CUDA"):
        sparc_b200.real_scan(torch.rand(1, 4, 3), torch.rand(1, 4, 3))


def test_module_api_matches_reference(golden):
    """Constructor, parameter/buffer names and shapes, init values under manual_seed(0) and the
    setters' validation, against the reference module (golden init.npz)."""
    import numpy as np
    import torch

    import sparc_b200

    d = golden("init")
    for W in (16, 64):
        torch.manual_seed(0)
        m = sparc_b200.SPARCMixer(W)
        sd = m.state_dict()
        ref_keys = sorted(k[len(f"w{W}_"):] for k in d.files if k.startswith(f"w{W}_"))
        assert sorted(sd.keys()) == ref_keys
        for k in ref_keys:
            np.testing.assert_array_equal(sd[k].double().numpy(), d[f"w{W}_{k}"])
    with pytest.raises(ValueError):
        sparc_b200.SPARCMixer(7)
    m = sparc_b200.SPARCMixer(8)
    with pytest.raises(ValueError):
        m.set_tiled_training_block_size(48)
    with pytest.raises(ValueError):
        m.set_controller_projection_dtype("fp16")
    with pytest.raises(ValueError):
        m.set_decode_backend("blocked8")
    m.set_scan_backend("chunk16")
    m.set_decode_backend("fused")
    m.prepare_inference()
    assert m._inference_fused


def test_torch_operators_registered():
    """The TORCH_LIBRARY registration exposes the C ABI as torch.ops.sparc_b200.* (schemas only:
    no compute without a GPU)."""
    from sparc_b200 import _build, torch_ops

    _build.build_torch_ops()
    ops = torch_ops.load()
    names = {"mixer_forward", "mixer_backward", "decode_step", "real_scan_forward", "real_scan_backward"}
    for n in names:
        assert hasattr(ops, n), n
    schema = str(ops.mixer_forward.default._schema)
    assert "Tensor x" in schema and "Tensor write_radial_response" in schema


def test_integration_stub_matches_the_header(lib, monkeypatch):
    """The ctypes stub a maintainer would add (tests/c_abi/sparc_ctypes_stub.py, quoted in the
    integration guide) has the header's struct layout and reads error messages correctly (loaded
    against the built library; no compute call is made)."""
    import ctypes
    import importlib.util

    from sparc_b200 import _lib

    monkeypatch.setenv("SPARC_B200_LIBRARY", _lib.LIB_PATH)
    spec = importlib.util.spec_from_file_location(
        "sparc_ctypes_stub", os.path.join(ROOT, "tests", "c_abi", "sparc_ctypes_stub.py"))
    ns = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ns)
    stub, ours = ns.SparcMixerFwdArgs, _lib.MixerFwdArgs
    assert [f[0] for f in stub._fields_] == [f[0] for f in ours._fields_]
    assert ctypes.sizeof(stub) == ctypes.sizeof(ours)
    for name, _ in ours._fields_:
        assert getattr(stub, name).offset == getattr(ours, name).offset, name
    assert ns.lib.sparc_mixer_forward(None, None) == -1  # SPARC_ERR_ARG
    assert ns.lib.sparc_last_error() == b"null args"
    assert ns.lib.sparc_mixer_carry_chunks(1 << 40, 0) == (1 << 40) // 8  # 64-bit return declared


def test_header_compiles_as_c_and_cxx_and_the_c_host_links(lib, tmp_path):
    """include/sparc_b200.h is plain C (and extern "C" under C++), and the C host program of the
    GPU test builds warning-free against it and links against the library (not run here)."""
    import subprocess

    from sparc_b200 import _lib

    inc = os.path.join(ROOT, "include")
    for compiler, lang in (("gcc", "c"), ("g++", "c++")):
        src = tmp_path / f"h.{lang}"
        src.write_text('#include "sparc_b200.h"\nint main(void) { return sparc_last_error() == 0; }\n')
        subprocess.run([compiler, "-x", lang, "-std=c11" if lang == "c" else "-std=c++17", "-Wall", "-Wextra",
                        "-Werror", "-pedantic", "-I", inc, "-fsyntax-only", str(src)], check=True)
    exe = tmp_path / "mixer_from_c"
    libdir = os.path.dirname(_lib.LIB_PATH)
    subprocess.run(["gcc", "-O2", "-Wall", "-Werror", "-o", str(exe), os.path.join(ROOT, "tests", "c_abi", "mixer_from_c.c"),
                    "-I", inc, "-I", "/usr/local/cuda/include", "-L", libdir, "-lsparc_b200",
                    "-L", "/usr/local/cuda/lib64", "-lcudart", "-lm", f"-Wl,-rpath,{libdir}"], check=True)
    assert exe.exists()


def test_entry_points_open_nvtx_ranges(lib, tmp_path):
    """Every compute entry point opens an NVTX range named after itself for the whole call (here
    calls rejected by their argument checks, so no device is needed), recorded by a test
    injection library (tests/c_abi/nvtx_recorder.c) that the library's NVTX client loads."""
    import json
    import subprocess
    import sys

    from sparc_b200 import _lib

    rec = tmp_path / "libnvtx_recorder.so"
    subprocess.run(["gcc", "-O2", "-Wall", "-Werror", "-shared", "-fPIC", "-o", str(rec),
                    os.path.join(ROOT, "tests", "c_abi", "nvtx_recorder.c"), "-I", "/usr/local/cuda/include"],
                   check=True)
    names = ["sparc_mixer_forward", "sparc_mixer_backward", "sparc_mixer_forward_noalloc", "sparc_decode_step",
             "sparc_real_scan_forward", "sparc_real_scan_backward", "sparc_rtrl_step", "sparc_rtrl_grad",
             "sparc_proj_gemm", "sparc_peer_allreduce"]
    code = (
        "import ctypes, json, sys\n"
        "lib = ctypes.CDLL(sys.argv[1])\n"
        "rcs = [getattr(lib, n)(None, None) for n in json.loads(sys.argv[3])]\n"
        "rec = ctypes.CDLL(sys.argv[2])\n"
        "rec.nvtx_recorder_log.restype = ctypes.c_char_p\n"
        "print(json.dumps({'rcs': rcs, 'log': rec.nvtx_recorder_log().decode()}))\n")
    env = dict(os.environ, NVTX_INJECTION64_PATH=str(rec))
    out = subprocess.run([sys.executable, "-c", code, _lib.LIB_PATH, str(rec), json.dumps(names)], env=env,
                         capture_output=True, text=True, timeout=120, check=True)
    res = json.loads(out.stdout.strip().splitlines()[-1])
    assert res["rcs"] == [-1] * len(names)  # each rejected: null args
    assert res["log"].split() == [x for n in names for x in (f"push:{n}", "pop")]


def test_state_dict_round_trips_with_the_reference_layout(golden):
    """Checkpoint / resume: a reference SPARCMixer state dict (its names, shapes and values, from
    the golden init.npz) loads strictly into ours and saves back unchanged, through torch.save."""
    import io

    import numpy as np
    import torch

    import sparc_b200

    d = golden("init")
    W = 64
    ref_sd = {k[len(f"w{W}_"):]: torch.tensor(d[k], dtype=torch.float32) for k in d.files if k.startswith(f"w{W}_")}
    torch.manual_seed(123)  # a different init, overwritten by the load
    m = sparc_b200.SPARCMixer(W)
    m.load_state_dict(ref_sd, strict=True)
    buf = io.BytesIO()
    torch.save(m.state_dict(), buf)
    buf.seek(0)
    m2 = sparc_b200.SPARCMixer(W)
    m2.load_state_dict(torch.load(buf), strict=True)
    for k, v in ref_sd.items():
        np.testing.assert_array_equal(m2.state_dict()[k].numpy(), v.numpy(), err_msg=k)


def test_rtrl_carry_api_matches_reference():
    """initialize_traces / initialize_carry (training/rtrl.py:25-46) and SPARCRTRLCell.initial_carry
    (layers.py:84-85) take the reference's positional arguments (..., dtype) and build the same
    shapes: modal traces [B, M], content [B, W, M], controllers [B, W + 1, M], complex64."""
    import inspect

    import torch

    import sparc_b200
    from sparc_b200 import rtrl

    assert list(inspect.signature(rtrl.initialize_traces).parameters)[:4] == ["batch_size", "input_size", "modes", "dtype"]
    assert list(inspect.signature(rtrl.initialize_carry).parameters)[:4] == ["batch_size", "input_size", "modes", "dtype"]
    state, tr = sparc_b200.initialize_carry(2, 3, 4, torch.complex128)
    assert state.shape == (2, 4) and state.dtype == torch.complex128
    shapes = {n: tuple(t.shape) for n, t in tr.items()}
    assert shapes["decay_log"] == (2, 4) and shapes["content_real"] == (2, 3, 4) and shapes["phase_controller"] == (2, 4, 4)
    assert set(shapes) == set(rtrl.TRACE_NAMES) and len(shapes) == 9
    cell = sparc_b200.SPARCRTRLCell(3, 4)
    assert list(inspect.signature(cell.initial_carry).parameters)[:3] == ["batch_size", "input_size", "dtype"]
    s2, tr2 = cell.initial_carry(2, 3, torch.complex64)
    assert s2.dtype == torch.complex64 and tr2["retention_controller"].shape == (2, 4, 4)


def test_missing_library_fails_loudly(tmp_path):
    """Without the built library every entry point raises (no CPU or Python fallback): a fresh
    process whose loader points at a missing file."""
    import subprocess
    import sys

    code = ("import torch, sparc_b200\n"
            "from sparc_b200 import _lib\n"
            f"_lib.LIB_PATH = {str(tmp_path / 'missing.so')!r}\n"
            "_lib.load_library.__defaults__ = (_lib.LIB_PATH,)\n"
            "try:\n"
            "    sparc_b200.real_scan_with_last(torch.rand(1, 4, 3), torch.rand(1, 4, 3))\n"
            "except RuntimeError as e:\n"
            "    print('raised:', e)\n"
            "try:\n"
            "    _lib.lib()\n"
            "except RuntimeError as e:\n"
            "    print('raised:', e)\n")
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("raised:")]
    assert len(lines) == 2 and "missing" in lines[1] and "no CPU or Python fallback" in lines[1]
