"""Build libflashmaxsim_sm100.so in-tree with nvcc for sm_100a (B200).

The library is plain CUDA C++ behind a C ABI (include/flash_maxsim_sm100.h);
Python reaches it through ctypes, so no torch headers are involved.

    python flash_maxsim_b200/build.py          # build if sources changed
    python flash_maxsim_b200/build.py --force  # always rebuild

(Run it as a script: importing the package itself loads the library.)
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_NAME = "libflashmaxsim_sm100.so"
LIB_PATH = PKG_DIR / LIB_NAME
SOURCES = [CSRC / "fm_capi.cu"]
DEPENDS = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [
    REPO_DIR / "include" / "flash_maxsim_sm100.h"
]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-shared",
    # IEEE division / square root and no contraction surprises: the INT8
    # quantiser must be bit-exact with the reference's torch formula.
    "-prec-div=true",
    "-prec-sqrt=true",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    p = Path(cuda_home) / "bin" / "nvcc"
    if p.exists():
        return str(p)
    raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(p.exists() and p.stat().st_mtime > t for p in DEPENDS)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the shared library if it is missing or older than its sources."""
    if not force and not needs_build():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *NVCC_FLAGS, *map(str, SOURCES), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose=True)
    print(path)


def load_build_module():
    """This module, loaded by file path without importing the package."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("_fm_build", Path(__file__))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod
