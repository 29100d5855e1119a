"""The tcgen05 (UMMA) descriptor encoders against CUTLASS's own bitfield definitions.

plastic_infer_b200/csrc/umma_desc.cuh encodes the shared-memory matrix descriptor and
the kind::f16 instruction descriptor with shifts. tests/native/umma_desc_check.cu fills
CUTLASS's cute::UMMA unions field by field for the same values and compares, on the host:
no GPU is involved. Skipped when nvcc or a CUTLASS include tree is not available.
"""

from __future__ import annotations

import pathlib
import shutil
import site
import subprocess

import pytest

HERE = pathlib.Path(__file__).resolve().parent
CSRC = HERE.parent / "plastic_infer_b200" / "csrc"


def _cutlass_include() -> pathlib.Path | None:
    roots = [pathlib.Path(p) for p in site.getsitepackages()]
    for root in roots:
        for rel in ("flashinfer/data/cutlass/include", "tilelang/3rdparty/cutlass/include"):
            cand = root / rel
            if (cand / "cute" / "arch" / "mma_sm100_desc.hpp").exists():
                return cand
    return None


def test_umma_descriptor_encoders_match_cutlass(tmp_path) -> None:
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    inc = _cutlass_include()
    if not pathlib.Path(nvcc).exists() or inc is None:
        pytest.skip("nvcc or the CUTLASS headers are not available")
    exe = tmp_path / "umma_desc_check"
    build = subprocess.run(
        [nvcc, "-std=c++17", "-Wno-deprecated-gpu-targets", f"-I{inc}", f"-I{CSRC}", "-o", str(exe),
         str(HERE / "native" / "umma_desc_check.cu")],
        capture_output=True, text=True, timeout=600)
    assert build.returncode == 0, build.stderr[-3000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and run.stdout.startswith("ok"), run.stdout + run.stderr
