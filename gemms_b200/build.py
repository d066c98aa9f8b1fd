"""Compile the sm_100a CUDA sources into the in-tree shared libraries.

``python -m gemms_b200.build`` (or ``__graft_entry__.build()``) runs nvcc on
``gemms_b200/csrc/*.cu`` and writes ``gemms_b200/lib/libgemms_b200.so`` (the C
ABI of ``include/gemms_moe.h``), then compiles ``csrc/torch_ops.cpp`` against
PyTorch's headers into ``gemms_b200/lib/libgemms_torch.so`` (the
``torch.ops.gemms_b200`` operators, which call the C ABI).  A library is
rebuilt only when one of its sources or headers is newer than it.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libgemms_b200.so")
TORCH_LIB = os.path.join(LIBDIR, "libgemms_torch.so")
TORCH_SRC = os.path.join(CSRC, "torch_ops.cpp")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         "-cudart", "shared", "-Xptxas", "-v"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def cuda_home() -> str:
    return os.path.dirname(os.path.dirname(os.path.realpath(nvcc())))


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(f) <= t for f in deps)


def up_to_date() -> bool:
    return _newer(LIB, _deps())


def _run(cmd: list[str], log_name: str, what: str) -> str:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    log = proc.stdout + proc.stderr
    with open(os.path.join(LIBDIR, log_name), "w") as f:
        f.write(" ".join(cmd) + "\n" + log)
    if proc.returncode != 0:
        raise RuntimeError(f"{what} failed ({proc.returncode}):\n{log[-6000:]}")
    return log


def build_torch_ops(force: bool = False) -> str:
    """torch.ops.gemms_b200.{moe, run}: g++ against the installed PyTorch,
    linked to libgemms_b200.so (found next to it at run time)."""
    deps = [TORCH_SRC, LIB] + glob.glob(os.path.join(ROOT, "include", "*.h"))
    if not force and _newer(TORCH_LIB, deps):
        return TORCH_LIB
    import torch
    from torch.utils import cpp_extension

    tdir = os.path.dirname(torch.__file__)
    inc = []
    for d in cpp_extension.include_paths() + [os.path.join(cuda_home(), "include"), os.path.join(ROOT, "include")]:
        inc += ["-I", d]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = TORCH_LIB + ".tmp"
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *inc, TORCH_SRC, "-o", tmp, "-L", LIBDIR, "-lgemms_b200", "-L", os.path.join(tdir, "lib"), "-lc10",
           "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-Wl,-rpath,$ORIGIN"]
    _run(cmd, "build_torch.log", "g++ (torch operators)")
    os.replace(tmp, TORCH_LIB)
    return TORCH_LIB


def build(force: bool = False, verbose: bool = False, torch_ops: bool = True) -> str:
    if force or not up_to_date():
        os.makedirs(LIBDIR, exist_ok=True)
        tmp = LIB + ".tmp"
        cmd = [nvcc(), *ARCH, *FLAGS, "-shared", "-I", os.path.join(ROOT, "include"), "-o", tmp, *sources()]
        log = _run(cmd, "build.log", "nvcc")
        if verbose:
            print(log)
        os.replace(tmp, LIB)
    if torch_ops:
        build_torch_ops(force=force)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
