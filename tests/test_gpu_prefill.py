"""GPU parity of paged prefill attention (pi_paged_prefill_attn and its tcgen05 twin
pi_paged_prefill_attn_tc; every case runs on both).

One request's q_len new tokens attend, straight from the page pool, to the first kv_len
tokens of their pages: causally from position q_start (the reference's is_causal path
at q_start == 0 and its dense offset mask otherwise) or non-causally. Tolerance is the
attention bar: |err| <= 2e-2 + 1e-2 |ref| against the oracle evaluated on exactly the
bf16/f16 values the kernel reads. Covered:
- the reference's own outputs (golden prefill.npz);
- G = 1/2/4/8/16, head_dim 64/128, pages of 16/32 tokens, f16;
- q_len not a multiple of a CTA's token block, kv_len not a multiple of the page;
- NaN in every unused slot of the last page;
- a strided q (fused QKV slice), an empty context;
- the reference algorithm run on the GPU (gather + repeat_interleave + SDPA).
"""

from __future__ import annotations

import pathlib

import numpy as np
import pytest
import torch

from oracle import paged_kv_oracle as orc
from plastic_infer_b200 import kernels
from tests.golden.inputs import PREFILL_CASES, prefill_inputs

pytestmark = pytest.mark.gpu
GOLD = pathlib.Path(__file__).resolve().parent / "golden"
DEV = torch.device("cuda", 0)
ATOL, RTOL = 2e-2, 1e-2


def _close(got: np.ndarray, ref: np.ndarray) -> None:
    err = np.abs(got - ref)
    bad = err > ATOL + RTOL * np.abs(ref)
    assert not bad.any(), f"max abs err {err.max():.3e}, {int(bad.sum())} of {bad.size} outside"


def _setup(q_len, kv_len, Hq, Hkv, D, S, dtype, seed, poison=False, k_rows=None, v_rows=None,
           q=None, table=None):
    """Device pools (physical) holding the context at `table`'s pages, plus the logical
    float32 copy the oracle reads (values exactly as stored in `dtype`)."""
    rng = np.random.default_rng(seed)
    npg = -(-kv_len // S)
    if table is None:
        P = npg + 5
        table = rng.permutation(P)[:npg].astype(np.int32)
    else:
        P = int(table.max()) + 2 if len(table) else 2
    if k_rows is None:
        k_rows = rng.standard_normal((kv_len, Hkv, D), dtype=np.float32)
        v_rows = rng.standard_normal((kv_len, Hkv, D), dtype=np.float32)
    if q is None:
        q = rng.standard_normal((q_len, Hq, D), dtype=np.float32)
    fill = np.nan if poison else 0.0
    kp = np.full((P, Hkv, S, D), fill, dtype=np.float32)
    vp = np.full((P, Hkv, S, D), fill, dtype=np.float32)
    for t in range(kv_len):
        kp[table[t // S], :, t % S] = k_rows[t]
        vp[table[t // S], :, t % S] = v_rows[t]
    kp_d = torch.from_numpy(kp).to(dtype).to(DEV)
    vp_d = torch.from_numpy(vp).to(dtype).to(DEV)
    q_d = torch.from_numpy(q).to(dtype).to(DEV)
    # what the kernel reads, back in float32 and in the reference's logical layout
    lk = kp_d.float().cpu().numpy().transpose(0, 1, 3, 2)
    lv = vp_d.float().cpu().numpy().transpose(0, 1, 3, 2)
    return q_d, kp_d, vp_d, torch.from_numpy(table).to(DEV), lk, lv, list(table)


IMPLS = ["mma", "tc"]  # mma.sync kernel, tcgen05 kernel (S and O in tensor memory)


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("case", PREFILL_CASES, ids=[c["name"] for c in PREFILL_CASES])
def test_prefill_matches_reference_golden(case: dict, impl: str) -> None:
    g = np.load(GOLD / "prefill.npz")
    n = case["name"]
    x = prefill_inputs(case)
    q, kp, vp, bt, lk, lv, table = _setup(case["q_len"], case["kv_len"], case["Hq"], case["Hkv"],
                                          case["D"], case["S"], torch.bfloat16, 0, k_rows=x["k"],
                                          v_rows=x["v"], q=x["q"], table=g[n + "__table"])
    out = kernels.paged_prefill_attention(q, kp, vp, bt, case["kv_len"], case["q_start"],
                                          case["causal"], impl=impl)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    ref = orc.paged_attention_prefill(q.float().cpu().numpy(), lk, lv, table, case["kv_len"],
                                      case["q_start"], case["causal"], case["S"])
    _close(got, ref)
    # and the reference's fp32 result itself, within bf16 input rounding
    assert np.abs(got - g[n + "__out"]).max() < 6e-2


CASES = [
    # (q_len, kv_len, q_start, causal, Hq, Hkv, D, S, dtype)
    (300, 700, 400, True, 32, 8, 128, 16, torch.bfloat16),    # 8B heads, chunked prefill
    (129, 129, 0, True, 32, 8, 128, 16, torch.bfloat16),      # first prefill, ragged block
    (70, 90, 20, True, 32, 4, 128, 16, torch.bfloat16),       # MoE heads (G = 8)
    (65, 200, 135, True, 8, 8, 64, 32, torch.float16),        # MHA, 32-token pages, f16
    (33, 51, 18, True, 32, 2, 128, 16, torch.bfloat16),       # G = 16
    (40, 77, 0, False, 8, 4, 64, 16, torch.bfloat16),         # non-causal, G = 2
    (5, 3, 0, False, 4, 2, 64, 16, torch.bfloat16),           # keys fewer than one page
]


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("q_len,kv_len,q_start,causal,Hq,Hkv,D,S,dtype", CASES)
def test_prefill_vs_oracle(q_len, kv_len, q_start, causal, Hq, Hkv, D, S, dtype, impl) -> None:
    q, kp, vp, bt, lk, lv, table = _setup(q_len, kv_len, Hq, Hkv, D, S, dtype, seed=q_len + kv_len,
                                          poison=True)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = kernels.paged_prefill_attention(q, kp, vp, bt, kv_len, q_start, causal, err=err, impl=impl)
    torch.cuda.synchronize()
    lk = np.nan_to_num(lk)  # the oracle reads only context rows; the NaNs are past kv_len
    lv = np.nan_to_num(lv)
    ref = orc.paged_attention_prefill(q.float().cpu().numpy(), lk, lv, table, kv_len, q_start,
                                      causal, S)
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert int(err.item()) == 0
    _close(got, ref)


# Larger shapes for the tcgen05 kernel: many 128-key tiles through the 2-stage ring,
# several query blocks per KV head, a q block that straddles q_len inside a warp.
TC_CASES = [
    # (q_len, kv_len, q_start, causal, Hq, Hkv, D, S, dtype)
    (1024, 4096, 3072, True, 32, 8, 128, 16, torch.bfloat16),   # chunk of a 4k prefill
    (1000, 1000, 0, True, 32, 8, 128, 16, torch.bfloat16),      # first prefill, ragged
    (77, 2500, 1200, False, 16, 16, 64, 32, torch.float16),     # non-causal, MHA, f16
    (200, 3000, 2800, True, 32, 2, 128, 32, torch.bfloat16),    # G = 16, 32-token pages
]


@pytest.mark.parametrize("q_len,kv_len,q_start,causal,Hq,Hkv,D,S,dtype", TC_CASES)
def test_prefill_tc_long_contexts_vs_oracle(q_len, kv_len, q_start, causal, Hq, Hkv, D, S,
                                            dtype) -> None:
    q, kp, vp, bt, lk, lv, table = _setup(q_len, kv_len, Hq, Hkv, D, S, dtype, seed=kv_len,
                                          poison=True)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = kernels.paged_prefill_attention(q, kp, vp, bt, kv_len, q_start, causal, err=err,
                                          impl="tc")
    torch.cuda.synchronize()
    ref = orc.paged_attention_prefill(q.float().cpu().numpy(), np.nan_to_num(lk),
                                      np.nan_to_num(lv), table, kv_len, q_start, causal, S)
    assert int(err.item()) == 0
    _close(out.float().cpu().numpy(), ref)


@pytest.mark.parametrize("impl", IMPLS)
def test_prefill_strided_q_out_param_and_empty_context(impl: str) -> None:
    q_len, kv_len, Hq, Hkv, D, S = 48, 100, 16, 4, 128, 16
    q, kp, vp, bt, lk, lv, table = _setup(q_len, kv_len, Hq, Hkv, D, S, torch.bfloat16, seed=7)
    qkv = torch.zeros((q_len, (Hq + 2 * Hkv) * D), dtype=torch.bfloat16, device=DEV)
    qkv[:, :Hq * D] = q.reshape(q_len, Hq * D)
    q_view = qkv[:, :Hq * D].view(q_len, Hq, D)
    out = torch.full((q_len, Hq, D), 7.0, dtype=torch.bfloat16, device=DEV)
    kernels.paged_prefill_attention(q_view, kp, vp, bt, kv_len, q_start=52, causal=True, out=out,
                                    impl=impl)
    ref = kernels.paged_prefill_attention(q, kp, vp, bt, kv_len, q_start=52, causal=True, impl=impl)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    # no context: zeros
    empty = kernels.paged_prefill_attention(q, kp, vp, bt[:0], 0, q_start=0, causal=True, impl=impl)
    torch.cuda.synchronize()
    assert int(torch.count_nonzero(empty)) == 0


@pytest.mark.parametrize("G", [1, 4, 16])
def test_prefill_tc_output_stays_inside_its_rows(G: int) -> None:
    # The tcgen05 kernel writes its output tile by TMA store, one 32-row box per warp. With
    # q_len ending inside a CTA's token block, rows of tokens past q_len must be dropped:
    # the buffer's rows after the output view keep their sentinel.
    Hkv, D, S = 2, 128, 16
    Hq = G * Hkv
    q_len, kv_len, q_start = 45, 300, 255
    q, kp, vp, bt, lk, lv, table = _setup(q_len, kv_len, Hq, Hkv, D, S, torch.bfloat16, seed=G)
    buf = torch.full((q_len + 40, Hq, D), 3.0, dtype=torch.bfloat16, device=DEV)
    out = kernels.paged_prefill_attention(q, kp, vp, bt, kv_len, q_start, True, out=buf[:q_len],
                                          impl="tc")
    torch.cuda.synchronize()
    assert bool((buf[q_len:] == 3.0).all())
    ref = orc.paged_attention_prefill(q.float().cpu().numpy(), lk, lv, table, kv_len, q_start,
                                      True, S)
    _close(out.float().cpu().numpy(), ref)
    # an output view whose base and token stride are not 16-byte multiples goes through a
    # temporary: same bits, and the columns around the view untouched
    wide = torch.full((q_len, Hq * D + 3), 5.0, dtype=torch.bfloat16, device=DEV)
    view = wide[:, 1:1 + Hq * D].view(q_len, Hq, D)
    kernels.paged_prefill_attention(q, kp, vp, bt, kv_len, q_start, True, out=view, impl="tc")
    torch.cuda.synchronize()
    assert torch.equal(view, out)
    assert bool((wide[:, 0] == 5.0).all()) and bool((wide[:, -2:] == 5.0).all())


@pytest.mark.parametrize("impl", IMPLS)
def test_prefill_matches_reference_algorithm_on_gpu(impl: str) -> None:
    # the reference's path (gather, repeat_interleave, SDPA with its offset mask) on the GPU
    import torch.nn.functional as F

    q_len, kv_len, q_start, Hq, Hkv, D, S = 96, 160, 64, 32, 8, 128, 16
    q, kp, vp, bt, lk, lv, table = _setup(q_len, kv_len, Hq, Hkv, D, S, torch.bfloat16, seed=11)
    out = kernels.paged_prefill_attention(q, kp, vp, bt, kv_len, q_start, True, impl=impl)
    kk = kp[bt.long()].permute(0, 2, 1, 3).reshape(-1, Hkv, D)[:kv_len]
    vv = vp[bt.long()].permute(0, 2, 1, 3).reshape(-1, Hkv, D)[:kv_len]
    G = Hq // Hkv
    qt = q.transpose(0, 1)[None]
    kt = kk.transpose(0, 1).repeat_interleave(G, dim=0)[None]
    vt = vv.transpose(0, 1).repeat_interleave(G, dim=0)[None]
    qpos = torch.arange(q_start, q_start + q_len, device=DEV)
    mask = torch.arange(kv_len, device=DEV)[None, :] <= qpos[:, None]
    am = torch.zeros(q_len, kv_len, dtype=q.dtype, device=DEV).masked_fill(~mask, float("-inf"))
    ref = F.scaled_dot_product_attention(qt, kt, vt, attn_mask=am[None, None])[0].transpose(0, 1)
    torch.cuda.synchronize()
    _close(out.float().cpu().numpy(), ref.float().cpu().numpy())
