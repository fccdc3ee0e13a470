"""Build libsparc_b200.so in-tree from csrc/*.cu with nvcc for sm_100a.

Each translation unit is compiled to an object in parallel (objects go to <repo>/_build/),
then linked into ``sparc_b200/libsparc_b200.so`` (the CUDA runtime is linked statically, so the
library only needs the driver). ``python -m sparc_b200._build`` rebuilds when a source changed.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libsparc_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I" + INCLUDE, "-I" + CSRC]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libsparc_b200")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in _deps())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)

    def compile_one(src):
        obj = os.path.join(BUILD, os.path.basename(src).replace(".cu", ".o"))
        cmd = [nvcc, *NVCC_FLAGS, *ARCH, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, file=sys.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = LIB + ".tmp"
    cmd = [nvcc, *ARCH, "-shared", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


TORCH_SRC = os.path.join(PKG, "csrc_torch", "torch_ops.cpp")
TORCH_LIB = os.path.join(PKG, "libsparc_b200_torch.so")


def build_torch_ops(force: bool = False, verbose: bool = False) -> str:
    """Build libsparc_b200_torch.so, the TORCH_LIBRARY registration of the C ABI
    (torch.ops.sparc_b200.*), with PyTorch's extension builder into _build/torch_ops and copy it
    in-tree. Its C-ABI symbols stay undefined: they resolve against libsparc_b200.so, which the
    loader (sparc_b200.torch_ops) opens with global visibility first."""
    deps = [TORCH_SRC, os.path.join(INCLUDE, "sparc_b200.h")]
    if not force and os.path.exists(TORCH_LIB) and all(os.path.getmtime(d) <= os.path.getmtime(TORCH_LIB) for d in deps):
        return TORCH_LIB
    import ctypes

    import torch.utils.cpp_extension as ce

    # the extension builder loads what it built: the C ABI must be resolvable first
    ctypes.CDLL(build(), mode=ctypes.RTLD_GLOBAL)
    bdir = os.path.join(BUILD, "torch_ops")
    os.makedirs(bdir, exist_ok=True)
    path = ce.load(name="sparc_b200_torch_ops", sources=[TORCH_SRC], extra_include_paths=[INCLUDE],
                   extra_cflags=["-O2"], build_directory=bdir, is_python_module=False, with_cuda=True,
                   verbose=verbose)
    built = os.path.join(bdir, "sparc_b200_torch_ops.so")
    if isinstance(path, str) and os.path.exists(path):
        built = path
    tmp = TORCH_LIB + ".tmp"
    shutil.copyfile(built, tmp)
    os.replace(tmp, TORCH_LIB)
    return TORCH_LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
    if "--torch" in sys.argv:
        print(build_torch_ops(force="--force" in sys.argv, verbose=True))
