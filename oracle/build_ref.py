"""Build the reference's own CUDA copy kernel into oracle/_ref/ (test infrastructure).

TEST INFRASTRUCTURE ONLY. Compiles oracle/ref_expert_copy.cu, which includes the
reference's src/plastic_infer/kernel/csrc/jit/fast_index_copy.cuh from the reference source
tree where it lies (nothing is copied), for sm_100a, into oracle/_ref/libref_expert_copy.so.
The library is git-ignored but travels with the working tree, so GPU tests and bench.py
can pin and time pi_expert_slot_copy against the reference kernel on a machine without the
reference tree. Skipped (returns None) when the reference tree is absent.

    python oracle/build_ref.py [--ref <plastic-infer checkout>]
"""

from __future__ import annotations

import argparse
import os
import pathlib
import shutil
import subprocess

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "_ref" / "libref_expert_copy.so"
# The reference checkout: $PLASTIC_INFER_REF, else a directory named `reference` beside
# this repository's root.
DEFAULT_REF = os.environ.get("PLASTIC_INFER_REF", str(HERE.parent.parent / "reference"))
CUH_DIR = pathlib.Path("src/plastic_infer/kernel/csrc/jit")


def build(ref: str = DEFAULT_REF, force: bool = False) -> pathlib.Path | None:
    jit = pathlib.Path(ref) / CUH_DIR
    if not (jit / "fast_index_copy.cuh").exists():
        return None
    src = HERE / "ref_expert_copy.cu"
    if OUT.exists() and not force and OUT.stat().st_mtime >= max(
            src.stat().st_mtime, (jit / "fast_index_copy.cuh").stat().st_mtime):
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC", "-cudart", "shared", "-I", str(jit), "-o", str(tmp), str(src)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=DEFAULT_REF)
    print(build(ap.parse_args().ref, force=True))
