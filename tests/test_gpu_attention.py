"""GPU parity of paged decode attention (row a2).

Tolerance: max-abs 2e-2 / rel 1e-2 against the reference's fp32
path on the same (bf16) inputs; fp32 pools (SIMT path) are held to 1e-4. Checked
against the reference's own outputs (golden attention.npz) and against the oracle on
larger seeded batches: ragged contexts, partial pages, empty requests, very long
single contexts (pieces merged across many warps), many tiny requests, GQA groups
1/4/8, head_dim 64/128/256, page sizes 16/32, fp16, NaN-poisoned unused slots.
"""

from __future__ import annotations

import pathlib
import zlib

import numpy as np
import pytest
import torch

from oracle import paged_kv_oracle as orc
from plastic_infer_b200 import _capi, kernels
from plastic_infer_b200.exec.attention import paged_attention_v1
from tests._helpers import assert_close, from_bits, logical_f32, physical_from_logical
from tests.golden.inputs import ATTENTION_CASES, attention_inputs

pytestmark = pytest.mark.gpu
GOLD = pathlib.Path(__file__).resolve().parent / "golden"
DEV = torch.device("cuda", 0)
ATOL, RTOL = 2e-2, 1e-2


def _tol(dtype: torch.dtype) -> tuple[float, float]:
    return (1e-4, 1e-4) if dtype == torch.float32 else (ATOL, RTOL)


def _tables_tensor(tables: list[list[int]], width: int | None = None) -> torch.Tensor:
    w = width or max(1, max(len(t) for t in tables))
    bt = torch.zeros((len(tables), w), dtype=torch.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
    return bt.to(DEV)


def _run(q, kp, vp, tables, ctx, **kw) -> np.ndarray:
    out = kernels.paged_decode_attention(q, kp, vp, _tables_tensor(tables),
                                         torch.tensor(ctx, dtype=torch.int32, device=DEV), **kw)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("case", ATTENTION_CASES, ids=[c["name"] for c in ATTENTION_CASES])
def test_attention_matches_reference_golden(case: dict) -> None:
    g = np.load(GOLD / "attention.npz")
    x = attention_inputs(case)
    if case["dtype"] == "bf16":
        q = from_bits(x["q_bits"]).to(DEV)
        kp = physical_from_logical(from_bits(x["k_bits"])).to(DEV)
        vp = physical_from_logical(from_bits(x["v_bits"])).to(DEV)
    else:
        q = torch.from_numpy(x["q"]).to(DEV)
        kp = physical_from_logical(torch.from_numpy(x["k"])).to(DEV)
        vp = physical_from_logical(torch.from_numpy(x["v"])).to(DEV)
    out = _run(q, kp, vp, x["tables"], x["ctx"])
    assert_close(out, g[case["name"] + "/out"], *_tol(q.dtype))


def _random_batch(seed: int, B: int, Hq: int, Hkv: int, D: int, S: int, ctx: list[int],
                  dtype: torch.dtype, extra_pages: int = 3):
    rng = np.random.default_rng(seed)
    npg = [-(-c // S) for c in ctx]
    P = sum(npg) + extra_pages
    perm = rng.permutation(P)
    tables, cur = [], 0
    for n in npg:
        tables.append([int(p) for p in perm[cur:cur + n]])
        cur += n
    q = torch.from_numpy(rng.standard_normal((B, Hq, D), dtype=np.float32)).to(dtype).to(DEV)
    kp = torch.from_numpy(rng.standard_normal((P, Hkv, S, D), dtype=np.float32)).to(dtype).to(DEV)
    vp = torch.from_numpy(rng.standard_normal((P, Hkv, S, D), dtype=np.float32)).to(dtype).to(DEV)
    return q, kp, vp, tables


def _oracle(q, kp, vp, tables, ctx, S) -> np.ndarray:
    return orc.paged_attention_decode(q.float().cpu().numpy(), logical_f32(kp), logical_f32(vp),
                                      tables, ctx, S)


CONFIGS = [
    # name, B, Hq, Hkv, D, S, ctx generator
    ("qwen3_8b_shape", 16, 32, 8, 128, 16, lambda r, B: r.integers(1, 2049, B)),
    ("qwen3_30b_a3b_shape", 12, 32, 4, 128, 16, lambda r, B: r.integers(1, 1500, B)),
    ("mha_d64_s32", 6, 8, 8, 64, 32, lambda r, B: r.integers(1, 700, B)),
    ("d256_g2", 5, 4, 2, 256, 16, lambda r, B: r.integers(1, 900, B)),
    ("one_long_context", 1, 32, 8, 128, 16, lambda r, B: np.array([20011])),
    ("many_tiny", 700, 8, 2, 128, 16, lambda r, B: r.integers(1, 40, B)),
    ("with_empty", 9, 32, 8, 128, 16, lambda r, B: np.array([0, 5, 0, 16, 17, 0, 300, 1, 0])),
]


@pytest.mark.parametrize("cfg", CONFIGS, ids=[c[0] for c in CONFIGS])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_attention_random_vs_oracle(cfg, dtype) -> None:
    name, B, Hq, Hkv, D, S, gen = cfg
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    ctx = [int(c) for c in gen(rng, B)]
    q, kp, vp, tables = _random_batch(7, B, Hq, Hkv, D, S, ctx, dtype)
    out = _run(q, kp, vp, tables, ctx)
    assert_close(out, _oracle(q, kp, vp, tables, ctx, S), ATOL, RTOL)


def test_attention_fp32_simt_path_vs_oracle() -> None:
    ctx = [1, 15, 16, 33, 250]
    q, kp, vp, tables = _random_batch(3, 5, 6, 3, 96, 16, ctx, torch.float32)
    out = _run(q, kp, vp, tables, ctx)
    assert_close(out, _oracle(q, kp, vp, tables, ctx, 16), 1e-4, 1e-4)


def test_attention_ignores_poisoned_unused_slots() -> None:
    # Unused pool pages and the tail of each last page hold NaN; the output must not.
    ctx = [17, 40, 3, 100]
    S = 16
    q, kp, vp, tables = _random_batch(11, 4, 32, 8, 128, S, ctx, torch.bfloat16, extra_pages=4)
    clean = _run(q, kp, vp, tables, ctx)
    used = torch.zeros(kp.shape[0], S, dtype=torch.bool)
    for t, n in zip(tables, ctx):
        for i, p in enumerate(t):
            used[p, :max(0, min(S, n - i * S))] = True
    mask = (~used).to(DEV)[:, None, :, None].expand_as(kp)
    kp = kp.masked_fill(mask, float("nan"))
    vp = vp.masked_fill(mask, float("nan"))
    poisoned = _run(q, kp, vp, tables, ctx)
    assert np.isfinite(poisoned).all()
    assert np.array_equal(poisoned, clean)


def test_attention_is_deterministic() -> None:
    ctx = [int(c) for c in np.random.default_rng(2).integers(1, 3000, 24)]
    q, kp, vp, tables = _random_batch(5, 24, 32, 8, 128, 16, ctx, torch.bfloat16)
    a = _run(q, kp, vp, tables, ctx)
    b = _run(q, kp, vp, tables, ctx)
    assert np.array_equal(a, b)


def test_attention_reports_bad_page_ids() -> None:
    ctx = [20]
    q, kp, vp, tables = _random_batch(6, 1, 8, 2, 128, 16, ctx, torch.bfloat16)
    tables[0][1] = kp.shape[0] + 5
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    _run(q, kp, vp, tables, ctx, err=err)
    assert int(err.item()) == _capi.PI_ERR_PAGE_RANGE


def test_attention_custom_scale_and_strided_q() -> None:
    ctx = [50, 7]
    q, kp, vp, tables = _random_batch(8, 2, 32, 8, 128, 16, ctx, torch.bfloat16)
    big = torch.zeros((2, 48 * 128), dtype=torch.bfloat16, device=DEV)
    big[:, :32 * 128] = q.view(2, -1)
    qs = big[:, :32 * 128].view(2, 32, 128)
    assert qs.stride(0) == 48 * 128
    out = _run(qs, kp, vp, tables, ctx, scale=0.05)
    ref = orc.paged_attention_decode(q.float().cpu().numpy(), logical_f32(kp), logical_f32(vp),
                                     tables, ctx, 16, scale=0.05)
    assert_close(out, ref, ATOL, RTOL)


@pytest.mark.parametrize("causal", [False, True])
def test_paged_attention_v1_decode_semantics(causal: bool) -> None:
    # Reference API on the store's logical view: [1, 1, Hq, D] query, list block table.
    ctx = [37]
    q, kp, vp, tables = _random_batch(9, 1, 8, 2, 128, 16, ctx, torch.bfloat16)
    out = paged_attention_v1(q.view(1, 1, 8, 128), kp.permute(0, 1, 3, 2), vp.permute(0, 1, 3, 2),
                             tables[0], 16, kv_num_tokens=37, causal=causal)
    # SDPA's causal mask is top-left aligned: one causal query sees only key 0.
    eff = [1] if causal else ctx
    ref = _oracle(q, kp, vp, tables, eff, 16)
    assert out.shape == (1, 1, 8, 128)
    assert_close(out[0].float().cpu().numpy(), ref, ATOL, RTOL)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fused_append_equals_copy_then_attend(dtype: torch.dtype) -> None:
    # One decode layer: write each request's new row at position ctx-1, then attend.
    ctx = [1, 17, 100, 513, 2048, 33, 16, 4000]
    S, Hq, Hkv, D = 16, 32, 8, 128
    q, kp, vp, tables = _random_batch(12, len(ctx), Hq, Hkv, D, S, ctx, dtype)
    g = torch.Generator().manual_seed(3)
    k_new = torch.randn((len(ctx), Hkv, D), generator=g).to(dtype).to(DEV)
    v_new = torch.randn((len(ctx), Hkv, D), generator=g).to(dtype).to(DEV)
    slots = [orc.slot_of(t, c - 1, S) for t, c in zip(tables, ctx)]
    slots[2] = -1  # a request without a new row this step
    slots[4] = orc.slot_of(tables[4], 700, S)  # a rewrite inside the context, not at its end
    slot_t = torch.tensor(slots, dtype=torch.int64, device=DEV)
    bt = _tables_tensor(tables)
    ctx_t = torch.tensor(ctx, dtype=torch.int32, device=DEV)
    kp2, vp2 = kp.clone(), vp.clone()
    kernels.kv_index_copy(kp, vp, k_new, v_new, slot_t)
    ref = kernels.paged_decode_attention(q, kp, vp, bt, ctx_t)
    out = kernels.paged_decode_attention(q, kp2, vp2, bt, ctx_t, k_new=k_new, v_new=v_new,
                                         slot_mapping=slot_t)
    torch.cuda.synchronize()
    assert torch.equal(kp2, kp) and torch.equal(vp2, vp)
    assert torch.equal(out, ref)
    # and against the oracle on the updated pool
    assert_close(out.float().cpu().numpy(), _oracle(q, kp, vp, tables, ctx, S), *_tol(dtype))
