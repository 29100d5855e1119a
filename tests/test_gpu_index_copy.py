"""GPU parity of the slot-mapping index-copy (row a1): bit-exact pool contents.

Against the reference's own results (golden: append_token + _write_kv_layer) and,
at larger sizes, against the oracle's write_kv_slots on the same seeded inputs.
All calls go through the C ABI (plastic_infer_b200.kernels -> pi_kv_index_copy).
"""

from __future__ import annotations

import pathlib

import numpy as np
import pytest
import torch

from oracle import paged_kv_oracle as orc
from plastic_infer_b200 import _capi, kernels
from tests._helpers import from_bits, logical_np

pytestmark = pytest.mark.gpu
GOLD = pathlib.Path(__file__).resolve().parent / "golden"
DEV = torch.device("cuda", 0)


def _batches_of_distinct(slots: np.ndarray) -> list[slice]:
    """Split a sequential write list where a slot repeats: writes within one launch
    must target distinct slots (launch order then gives last-write-wins)."""
    out, seen, start = [], set(), 0
    for i, s in enumerate(slots.tolist()):
        if s in seen:
            out.append(slice(start, i))
            seen, start = set(), i
        seen.add(s)
    out.append(slice(start, len(slots)))
    return out


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_index_copy_matches_reference_golden(dtype: str) -> None:
    g = np.load(GOLD / f"index_copy_{dtype}.npz")
    P, H, D, S = g["k_pages"].shape
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    kp = torch.zeros((P, H, S, D), dtype=tdt, device=DEV)
    vp = torch.zeros_like(kp)
    conv = from_bits if dtype == "bf16" else torch.from_numpy
    k_new = conv(g["k_new"]).to(DEV)
    v_new = conv(g["v_new"]).to(DEV)
    slots = torch.from_numpy(g["slots"]).to(DEV)
    batches = _batches_of_distinct(g["slots"])
    assert len(batches) == 2  # appends, then the _write_kv_layer overwrite pass
    for sl in batches:
        kernels.kv_index_copy(kp, vp, k_new[sl], v_new[sl], slots[sl])
    torch.cuda.synchronize()
    assert np.array_equal(logical_np(kp), g["k_pages"])
    assert np.array_equal(logical_np(vp), g["v_pages"])


def _rand_rows(rng: np.random.Generator, shape, dtype: torch.dtype) -> torch.Tensor:
    return torch.from_numpy(rng.standard_normal(shape, dtype=np.float32)).to(dtype)


@pytest.mark.parametrize("B", [1, 64, 512, 4096])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_index_copy_random_vs_oracle(B: int, dtype: torch.dtype) -> None:
    # C2 geometry (16-token pages, 8 KV heads, head_dim 128) on a 2048-page pool.
    P, H, S, D = 2048, 8, 16, 128
    rng = np.random.default_rng(B)
    init = _rand_rows(rng, (P, H, S, D), dtype)
    kp = init.to(DEV)
    vp = (init * 2).to(DEV)
    slots = rng.permutation(P * S)[:B].astype(np.int64)
    k_new = _rand_rows(rng, (B, H, D), dtype)
    v_new = _rand_rows(rng, (B, H, D), dtype)
    kernels.kv_index_copy(kp, vp, k_new.to(DEV), v_new.to(DEV), torch.from_numpy(slots).to(DEV))
    torch.cuda.synchronize()
    view = (lambda t: t.view(torch.int16).numpy()) if dtype != torch.float32 else (lambda t: t.numpy())
    ek = view(init.permute(0, 1, 3, 2).contiguous()).copy()
    ev = view((init * 2).permute(0, 1, 3, 2).contiguous()).copy()
    orc.write_kv_slots(ek, ev, view(k_new), view(v_new), slots, S)
    got_k = view(kp.permute(0, 1, 3, 2).contiguous().cpu())
    got_v = view(vp.permute(0, 1, 3, 2).contiguous().cpu())
    assert np.array_equal(got_k, ek)
    assert np.array_equal(got_v, ev)


def test_index_copy_padding_and_out_of_range() -> None:
    P, H, S, D = 8, 2, 16, 64
    kp = torch.zeros((P, H, S, D), dtype=torch.bfloat16, device=DEV)
    vp = torch.zeros_like(kp)
    new = torch.ones((4, H, D), dtype=torch.bfloat16, device=DEV)
    slots = torch.tensor([-1, 5, P * S, 17], dtype=torch.int64, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    kernels.kv_index_copy(kp, vp, new, new, slots, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == _capi.PI_ERR_SLOT_RANGE
    lg = kp.permute(0, 1, 3, 2).float().cpu()
    assert lg[0, :, :, 5].eq(1).all() and lg[1, :, :, 1].eq(1).all()
    assert float(lg.sum()) == 2 * H * D  # nothing else written


def test_index_copy_strided_source_fused_qkv() -> None:
    # k/v as column slices of a fused [B, (Hq + 2*Hkv) * D] projection output.
    P, Hq, H, S, D, B = 64, 32, 8, 16, 128, 48
    rng = np.random.default_rng(5)
    qkv = _rand_rows(rng, (B, (Hq + 2 * H) * D), torch.bfloat16).to(DEV)
    k = qkv[:, Hq * D:(Hq + H) * D].view(B, H, D)
    v = qkv[:, (Hq + H) * D:].view(B, H, D)
    assert k.stride(0) == (Hq + 2 * H) * D
    kp = torch.zeros((P, H, S, D), dtype=torch.bfloat16, device=DEV)
    vp = torch.zeros_like(kp)
    slots = torch.from_numpy(rng.permutation(P * S)[:B].astype(np.int64)).to(DEV)
    kernels.kv_index_copy(kp, vp, k, v, slots)
    pages, offs = slots // S, slots % S
    assert torch.equal(kp[pages, :, offs, :], k)
    assert torch.equal(vp[pages, :, offs, :], v)


def test_index_copy_misaligned_falls_back_to_narrow_vectors() -> None:
    # head_dim 3 in fp16: 6-byte rows -> 2-byte path; still bit-exact.
    P, H, S, D, B = 4, 3, 4, 3, 7
    kp = torch.zeros((P, H, S, D), dtype=torch.float16, device=DEV)
    vp = torch.zeros_like(kp)
    new = torch.randn((B, H, D), dtype=torch.float16, device=DEV)
    slots = torch.tensor([0, 3, 4, 9, 10, 14, 15], dtype=torch.int64, device=DEV)
    kernels.kv_index_copy(kp, vp, new, -new, slots)
    assert torch.equal(kp[slots // S, :, slots % S, :], new)
    assert torch.equal(vp[slots // S, :, slots % S, :], -new)


# Geometries that reach every launch shape of the kernel: one chunk per token (a single
# KV head, where a pass of two chunks spans two tokens), a partial last chunk (3 heads x
# 10 vectors), rows whose vector count is not a power of two (division path), one chunk
# per warp (small launches), two chunks per pass of one token (the whole 36-layer step in
# one launch) and a grid-stride loop beyond one wave (65,536 tokens).
GEOMETRIES = [
    # name, pages, kv_heads, page_size, head_dim, dtype, tokens
    ("c4_four_heads", 512, 4, 16, 128, torch.bfloat16, 128),
    ("one_head", 256, 1, 16, 128, torch.bfloat16, 300),
    ("one_head_two_tokens_per_pass", 256, 1, 16, 128, torch.bfloat16, 3000),
    ("three_chunks_per_token", 512, 3, 16, 128, torch.bfloat16, 1500),
    ("d96_rows_of_12_vectors", 256, 8, 16, 96, torch.bfloat16, 200),
    ("h3_d80_partial_chunk", 256, 3, 16, 80, torch.float16, 333),
    ("d64_page32", 256, 8, 32, 64, torch.bfloat16, 1000),
    ("f32_d64", 512, 2, 16, 64, torch.float32, 777),
    ("whole_step_36_layers", 4096, 8, 16, 128, torch.bfloat16, 36 * 64),
    ("large_65536", 8192, 8, 16, 128, torch.bfloat16, 65536),
]


@pytest.mark.parametrize("geom", GEOMETRIES, ids=[g[0] for g in GEOMETRIES])
def test_index_copy_geometries_vs_oracle(geom) -> None:
    name, P, H, S, D, dtype, B = geom
    rng = np.random.default_rng(len(name) * 7919 + B)
    init_k = _rand_rows(rng, (P, H, S, D), dtype)
    init_v = _rand_rows(rng, (P, H, S, D), dtype)
    kp, vp = init_k.to(DEV), init_v.to(DEV)
    slots = rng.permutation(P * S)[:B].astype(np.int64)
    slots[rng.random(B) < 0.05] = -1  # some padding tokens
    k_new = _rand_rows(rng, (B, H, D), dtype)
    v_new = _rand_rows(rng, (B, H, D), dtype)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    kernels.kv_index_copy(kp, vp, k_new.to(DEV), v_new.to(DEV), torch.from_numpy(slots).to(DEV),
                          err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    view = (lambda t: t.view(torch.int16).numpy()) if dtype != torch.float32 else (lambda t: t.numpy())
    ek = view(init_k.permute(0, 1, 3, 2).contiguous()).copy()
    ev = view(init_v.permute(0, 1, 3, 2).contiguous()).copy()
    orc.write_kv_slots(ek, ev, view(k_new), view(v_new), slots, S)
    assert np.array_equal(view(kp.permute(0, 1, 3, 2).contiguous().cpu()), ek)
    assert np.array_equal(view(vp.permute(0, 1, 3, 2).contiguous().cpu()), ev)


def test_index_copy_duplicate_slots_write_one_of_the_rows() -> None:
    # Duplicate slots in one launch: each 16-byte piece holds the bytes of one of the
    # duplicates (which one is unspecified); every other slot is exact.
    P, H, S, D, B = 64, 8, 16, 128, 96
    rng = np.random.default_rng(3)
    slots = rng.permutation(P * S)[:B].astype(np.int64)
    slots[50:60] = slots[0:10]
    kp = torch.zeros((P, H, S, D), dtype=torch.bfloat16, device=DEV)
    vp = torch.zeros_like(kp)
    k_new = _rand_rows(rng, (B, H, D), torch.bfloat16).to(DEV)
    v_new = _rand_rows(rng, (B, H, D), torch.bfloat16).to(DEV)
    st = torch.from_numpy(slots).to(DEV)
    kernels.kv_index_copy(kp, vp, k_new, v_new, st)
    got_k = kp[st // S, :, st % S, :].view(B, -1, 8)   # 16-byte pieces
    got_v = vp[st // S, :, st % S, :].view(B, -1, 8)
    kk, vv = k_new.view(B, -1, 8), v_new.view(B, -1, 8)
    for i in range(B):
        j = i - 50 if 50 <= i < 60 else (i + 50 if i < 10 else i)
        for got, src in ((got_k, kk), (got_v, vv)):
            piece_ok = (got[i] == src[i]).all(-1) | (got[i] == src[j]).all(-1)
            assert bool(piece_ok.all()), f"token {i}"
            if j == i:
                assert torch.equal(got[i], src[i])
