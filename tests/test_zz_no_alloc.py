"""The allocation-free attention entry point agrees with the workspace entry point.

pi_paged_decode_attn_noalloc serves callers that cannot allocate device memory
while decoding (a C-ABI-only host loop without a CUDA allocator, or an engine whose
memory planner gave every free byte to the page pool and the weights). It keeps its
split-KV scratch in one array compiled into the library instead of a caller-provided
workspace. This test calls it through the C ABI twice in a row, on batches that make
the kernel cut contexts across warps and merge the pieces (the part that uses the
scratch), and checks each result against pi_paged_decode_attn with a workspace,
within the attention tolerance used by the other GPU tests (2e-2 abs / 1e-2 rel).
The file sorts last so that a run stopping at the first failure has run every
other test first; it also passes on its own in a fresh process.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from plastic_infer_b200 import _capi, kernels

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
ATOL, RTOL = 2e-2, 1e-2


def _batch(seed: int, ctx: list[int], Hq=32, Hkv=8, D=128, S=16, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    npg = [-(-c // S) for c in ctx]
    P = sum(npg) + 2
    perm = torch.randperm(P, generator=g)
    bt = torch.zeros((len(ctx), max(npg)), dtype=torch.int32)
    cur = 0
    for i, n in enumerate(npg):
        bt[i, :n] = perm[cur:cur + n].to(torch.int32)
        cur += n
    q = torch.randn((len(ctx), Hq, D), generator=g).to(dtype).to(DEV)
    kp = torch.randn((P, Hkv, S, D), generator=g).to(dtype).to(DEV)
    vp = torch.randn((P, Hkv, S, D), generator=g).to(dtype).to(DEV)
    return q, kp, vp, bt.to(DEV), torch.tensor(ctx, dtype=torch.int32, device=DEV)


def _noalloc(q, kp, vp, bt, ctx_lens, out, err=None) -> int:
    B, Hq, D = q.shape
    P, Hkv, S, _ = kp.shape
    lib = _capi.load()
    return lib.pi_paged_decode_attn_noalloc(
        out.data_ptr(), q.data_ptr(), kp.data_ptr(), vp.data_ptr(), bt.data_ptr(), bt.stride(0),
        ctx_lens.data_ptr(), B, Hq, Hkv, D, S, P, 1.0 / math.sqrt(D), kernels.dtype_code(q.dtype),
        q.stride(0), out.stride(0), None if err is None else err.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


def _check(out: torch.Tensor, ref: torch.Tensor) -> None:
    o = out.float().cpu().numpy()
    r = ref.float().cpu().numpy()
    assert np.isfinite(o).all()
    bad = np.abs(o - r) > ATOL + RTOL * np.abs(r)
    assert not bad.any(), f"max abs diff {np.abs(o - r).max():.3e}"


def test_noalloc_matches_workspace_entry_point_two_calls_in_a_row() -> None:
    # call 1: ragged batch; call 2: a different batch (longer contexts, so more warps
    # share each (request, head) and the merge reads more partials from the scratch).
    cases = [(1, [513, 4096, 17, 1, 2500, 800, 3001, 64]),
             (2, [20011, 7, 9000, 150])]
    for seed, ctx in cases:
        q, kp, vp, bt, ctx_lens = _batch(seed, ctx)
        ref = kernels.paged_decode_attention(q, kp, vp, bt, ctx_lens)
        out = torch.full_like(ref, float("nan"))
        err = torch.zeros(1, dtype=torch.int32, device=DEV)
        rc = _noalloc(q, kp, vp, bt, ctx_lens, out, err)
        assert rc == _capi.PI_OK, _capi.error_string(rc)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        _check(out, ref)


def test_noalloc_rejects_requests_beyond_its_scratch() -> None:
    # head_dim 256 needs ~20 MB of partials on a B200, more than the 12 MiB array.
    q, kp, vp, bt, ctx_lens = _batch(3, [40, 70], Hq=8, Hkv=2, D=256)
    out = torch.empty_like(q)
    need = kernels.workspace_bytes(2, 8, 2, 256)
    assert need > _capi.NOALLOC_SCRATCH_BYTES
    rc = _noalloc(q, kp, vp, bt, ctx_lens, out)
    assert rc == _capi.PI_ERR_SCRATCH_LIMIT
    assert "scratch" in _capi.error_string(rc)


def test_noalloc_serves_simt_path_shapes_without_a_scratch_limit() -> None:
    # fp32 pools at head_dim 256 run on the generic SIMT path, which uses no scratch, so
    # the size limit does not apply even though the fast path's need would exceed it.
    q, kp, vp, bt, ctx_lens = _batch(4, [40, 70, 1], Hq=8, Hkv=2, D=256, dtype=torch.float32)
    ref = kernels.paged_decode_attention(q, kp, vp, bt, ctx_lens)
    out = torch.full_like(ref, float("nan"))
    rc = _noalloc(q, kp, vp, bt, ctx_lens, out)
    assert rc == _capi.PI_OK, _capi.error_string(rc)
    torch.cuda.synchronize()
    assert torch.allclose(out, ref, atol=1e-5, rtol=1e-5)
