"""Build libplastic_kv.so in-tree with nvcc for sm_100a.

The reference JIT-compiles its one CUDA kernel per template combination into
~/.cache (src/plastic_infer/kernel/jit.py:87-124). Here the whole C ABI is one
shared library built ahead of time inside the package directory, so the built
file travels with the source tree and is the file the tests and the benchmark load.

    python -m plastic_infer_b200._build          # build (skips when up to date)
    python -m plastic_infer_b200._build --force  # rebuild
"""

from __future__ import annotations

import os
import pathlib
import shutil
import subprocess
import sys

PKG_DIR = pathlib.Path(__file__).resolve().parent
CSRC_DIR = PKG_DIR / "csrc"
INCLUDE_DIR = PKG_DIR.parent / "include"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libplastic_kv.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-shared",
    "-Xcompiler",
    "-fPIC",
    "-cudart",
    "shared",
]


def _sources() -> list[pathlib.Path]:
    return sorted(CSRC_DIR.glob("*.cu"))


def _inputs() -> list[pathlib.Path]:
    return _sources() + sorted(CSRC_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


def nvcc_path() -> str:
    nvcc = shutil.which("nvcc")
    if nvcc is None:
        cand = pathlib.Path("/usr/local/cuda/bin/nvcc")
        if cand.exists():
            return str(cand)
        raise RuntimeError("nvcc not found: cannot build libplastic_kv.so")
    return nvcc


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    built = LIB_PATH.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in _inputs())


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    """Compile every .cu under csrc/ into one shared library; return its path."""
    if not force and up_to_date():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, "-o", str(tmp), *map(str, _sources())]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        tmp.unlink(missing_ok=True)
        raise RuntimeError(f"nvcc failed building libplastic_kv.so:\n{proc.stderr[-6000:]}")
    if verbose and proc.stderr:
        print(proc.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB_PATH)
