"""GPU parity of the MoE expert-slot copy (pi_expert_slot_copy).

Rows move from pinned host banks (read through their device alias) into device slot
caches, for every bank in one launch. The result must equal, byte for byte:
- the oracle's numpy row copy;
- the reference's own fused multi-bank kernel (fast_index_copy.cuh), compiled from the
  reference tree into oracle/_ref/ by oracle/build_ref.py. This part is skipped when that
  library was not built.
Covered: int32 and int64 indices, a device-side valid length shorter than the index
arrays, row sizes that are not multiples of the 4 KiB work chunk, CUDA-graph replays with
new indices and lengths, and the error paths (misaligned bank, negative index).
"""

from __future__ import annotations

import ctypes
import pathlib

import numpy as np
import pytest
import torch

from oracle import paged_kv_oracle as orc
from plastic_infer_b200 import _capi, kernels

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
REF_LIB = pathlib.Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libref_expert_copy.so"
ROW_BYTES = (6144, 5008, 48)   # 1.5 chunks, a ragged last chunk, a sub-chunk row
EXPERTS, SLOTS = 24, 16


def _banks(seed: int = 0):
    rng = np.random.default_rng(seed)
    src = [torch.from_numpy(rng.integers(0, 256, size=(EXPERTS, rb), dtype=np.uint8)).pin_memory()
           for rb in ROW_BYTES]
    dst = [torch.zeros((SLOTS, rb), dtype=torch.uint8, device=DEV) for rb in ROW_BYTES]
    desc = dict(
        dst_ptrs=torch.tensor([d.data_ptr() for d in dst], dtype=torch.int64, device=DEV),
        src_ptrs=torch.tensor([s.data_ptr() for s in src], dtype=torch.int64, device=DEV),
        feat_bytes=torch.tensor(list(ROW_BYTES), dtype=torch.int64, device=DEV),
    )
    return src, dst, desc


def _ref_lib():
    if not REF_LIB.exists():
        return None
    lib = ctypes.CDLL(str(REF_LIB))
    lib.ref_fast_index_copy_multi_launch.argtypes = [ctypes.c_void_p] * 5 + [
        ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    lib.ref_fast_index_copy_multi_launch.restype = None
    return lib


@pytest.mark.parametrize("idx_dtype", [torch.int32, torch.int64])
def test_expert_copy_matches_oracle_and_reference_kernel(idx_dtype: torch.dtype) -> None:
    src, dst, desc = _banks()
    rng = np.random.default_rng(1)
    L = 10
    dst_idx = rng.permutation(SLOTS)[:L]
    src_idx = rng.integers(0, EXPERTS, size=L)
    n = 7  # valid length below the index arrays' length
    di = torch.from_numpy(dst_idx).to(idx_dtype).to(DEV)
    si = torch.from_numpy(src_idx).to(idx_dtype).to(DEV)
    num = torch.tensor([n], dtype=torch.int64, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    kernels.expert_slot_copy(desc["dst_ptrs"], desc["src_ptrs"], desc["feat_bytes"], di, si, num,
                             err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    expect = [np.zeros((SLOTS, rb), dtype=np.uint8) for rb in ROW_BYTES]
    orc.expert_slot_copy(expect, [s.numpy() for s in src], dst_idx, src_idx, n)
    for got, exp in zip(dst, expect):
        assert np.array_equal(got.cpu().numpy(), exp)
    lib = _ref_lib()
    if lib is None:
        pytest.skip("reference kernel not built (oracle/build_ref.py needs the reference tree)")
    _, dst_r, desc_r = _banks()
    lib.ref_fast_index_copy_multi_launch(
        desc_r["dst_ptrs"].data_ptr(), desc_r["src_ptrs"].data_ptr(), desc_r["feat_bytes"].data_ptr(),
        di.data_ptr(), si.data_ptr(), L, num.data_ptr(), len(ROW_BYTES),
        1 if idx_dtype == torch.int32 else 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    for ours, theirs in zip(dst, dst_r):
        assert torch.equal(ours, theirs)


def test_expert_copy_graph_replays_with_new_indices() -> None:
    src, dst, desc = _banks(2)
    L = 12
    di = torch.zeros(L, dtype=torch.int32, device=DEV)
    si = torch.zeros(L, dtype=torch.int32, device=DEV)
    num = torch.zeros(1, dtype=torch.int64, device=DEV)
    kernels.expert_slot_copy(desc["dst_ptrs"], desc["src_ptrs"], desc["feat_bytes"], di, si, num)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        kernels.expert_slot_copy(desc["dst_ptrs"], desc["src_ptrs"], desc["feat_bytes"], di, si, num)
    expect = [np.zeros((SLOTS, rb), dtype=np.uint8) for rb in ROW_BYTES]
    rng = np.random.default_rng(3)
    for n in (3, 12, 0, 9):
        d = rng.permutation(SLOTS)[:L]
        s = rng.integers(0, EXPERTS, size=L)
        di.copy_(torch.from_numpy(d).to(torch.int32))
        si.copy_(torch.from_numpy(s).to(torch.int32))
        num.fill_(n)
        graph.replay()
        orc.expert_slot_copy(expect, [x.numpy() for x in src], d, s, n)
    torch.cuda.synchronize()
    for got, exp in zip(dst, expect):
        assert np.array_equal(got.cpu().numpy(), exp)
    del graph


def test_expert_copy_error_paths() -> None:
    src, dst, desc = _banks(4)
    di = torch.tensor([1, -1, 3], dtype=torch.int64, device=DEV)
    si = torch.tensor([0, 5, 2], dtype=torch.int64, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    kernels.expert_slot_copy(desc["dst_ptrs"], desc["src_ptrs"], desc["feat_bytes"], di, si, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == _capi.PI_ERR_SLOT_RANGE
    expect = [np.zeros((SLOTS, rb), dtype=np.uint8) for rb in ROW_BYTES]
    orc.expert_slot_copy(expect, [x.numpy() for x in src], np.array([1, 3]), np.array([0, 2]))
    for got, exp in zip(dst, expect):
        assert np.array_equal(got.cpu().numpy(), exp)
    # a bank whose row size is not a multiple of 16 bytes is skipped and reported
    bad = desc["feat_bytes"].clone()
    bad[2] = 40
    err.zero_()
    dst[2].zero_()
    kernels.expert_slot_copy(desc["dst_ptrs"], desc["src_ptrs"], bad, di[:1], si[:1], err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == _capi.PI_ERR_MISALIGNED
    assert int(torch.count_nonzero(dst[2])) == 0
