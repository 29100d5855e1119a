"""GPU parity of the page moves and the host KV store (row a3) and the store API (a4).

Bit-exact against the reference's own sink_completed_chunks / load_prefix results
(golden store_*.npz) and against the oracle's sink/load restatement; plus the
reference's KV-store test scenarios (tests/test_kv_store.py of plastic-infer) run
on a CUDA pool through this package.
"""

from __future__ import annotations

import pathlib

import numpy as np
import pytest
import torch

from oracle import paged_kv_oracle as orc
from plastic_infer_b200 import _capi, kernels
from plastic_infer_b200.kv import KVConfig, KVStore
from tests._helpers import from_bits, logical_np, to_bits
from tests.golden.inputs import token_kv

pytestmark = pytest.mark.gpu
GOLD = pathlib.Path(__file__).resolve().parent / "golden"
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("ppg", [1, 4])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_page_gather_scatter_roundtrip(ppg: int, dtype: torch.dtype) -> None:
    P, H, S, D, n = 300, 8, 16, 128, 64
    g = torch.Generator().manual_seed(ppg)
    pool = torch.randn((P, H, S, D), generator=g).to(dtype).to(DEV)
    ids = torch.randperm(P, generator=g)[:n].to(torch.int32)
    staging = torch.empty((n * H * S * D,), dtype=dtype, device=DEV)
    kernels.page_gather(pool, ids.to(DEV), staging, pages_per_group=ppg)
    # expected staging layout [n/ppg, H, ppg, S, D]
    exp = pool.cpu()[ids.long()].view(n // ppg, ppg, H, S, D).permute(0, 2, 1, 3, 4).contiguous()
    assert torch.equal(staging.cpu().view_as(exp), exp)
    # scatter into other pages of a fresh pool and read back
    dst_ids = torch.randperm(P, generator=g)[:n].to(torch.int32)
    pool2 = torch.zeros_like(pool)
    kernels.page_scatter(staging, dst_ids.to(DEV), pool2, pages_per_group=ppg)
    assert torch.equal(pool2.cpu()[dst_ids.long()], pool.cpu()[ids.long()])
    untouched = torch.ones(P, dtype=torch.bool)
    untouched[dst_ids.long()] = False
    assert pool2.cpu()[untouched].eq(0).all()


def test_page_moves_report_bad_ids() -> None:
    pool = torch.zeros((4, 2, 16, 64), dtype=torch.bfloat16, device=DEV)
    staging = torch.zeros(2 * 2 * 16 * 64, dtype=torch.bfloat16, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    kernels.page_gather(pool, torch.tensor([1, 9], dtype=torch.int32, device=DEV), staging, err=err)
    assert int(err.item()) == _capi.PI_ERR_PAGE_RANGE


def test_paged_kv_gather_matches_oracle() -> None:
    P, H, S, D = 40, 4, 16, 64
    pool = torch.randn((P, H, S, D), dtype=torch.bfloat16, device=DEV)
    table = [7, 3, 30, 12]
    out = kernels.paged_kv_gather(pool, torch.tensor(table, dtype=torch.int32, device=DEV), 57)
    lg = logical_np(pool)
    ek, _ = orc.gather_paged_kv(lg, lg, table, S, 57)
    assert np.array_equal(to_bits(out), ek)


def _store(dtype: torch.dtype, L=2, H=2, D=4, S=4, ppc=2, P=64, hc=8) -> KVStore:
    return KVStore(KVConfig(n_layers=L, n_kv_heads=H, head_dim=D, page_size=S,
                            pages_per_chunk=ppc, max_pages=P, max_host_chunks=hc, dtype=dtype,
                            device=DEV))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_store_sink_and_load_match_reference_golden(dtype: str) -> None:
    g = np.load(GOLD / f"store_{dtype}.npz")
    L, H, D, S, ppc, P = (int(g[k]) for k in ("L", "H", "D", "S", "ppc", "P"))
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    store = _store(tdt, L, H, D, S, ppc, P)
    ntok = len(g["tokens"])
    k, v = token_kv(21 if dtype == "f32" else 22, ntok, L, H, D, dtype)
    kt = torch.from_numpy(k).to(tdt).to(DEV)
    vt = torch.from_numpy(v).to(tdt).to(DEV)
    c1 = store.new_request()
    for t in range(ntok):
        c1.append_token(kt[t], vt[t])
    c1.set_token_ids([int(x) for x in g["tokens"]])
    assert store.sink_completed_chunks(c1) == int(g["sunk"])
    assert [k.full_key.hex() for k in c1.chunk_keys] == list(g["keys_hex"])
    assert np.array_equal(np.asarray([c1.get_block_table_for_layer(l) for l in range(L)]),
                          g["c1_tables"])
    conv = to_bits if dtype == "bf16" else (lambda t: t.cpu().numpy())
    for c, key in enumerate(c1.chunk_keys):
        hk, hv = store._host_cache[key.full_key]
        assert hk.shape == (L, H, D, S * ppc)
        assert np.array_equal(conv(hk.contiguous()), g["host_k"][c])
        assert np.array_equal(conv(hv.contiguous()), g["host_v"][c])
    store.free_request(c1)
    c2 = store.new_request()
    matched, keys = store.load_prefix(c2, [int(x) for x in g["tokens"]])
    assert matched == int(g["matched"]) and c2.length == int(g["c2_length"])
    tables = np.asarray([c2.get_block_table_for_layer(l) for l in range(L)])
    assert np.array_equal(tables, g["c2_tables"])
    assert store.gpu.allocator.free_pages == int(g["free_after_load"])
    for layer in range(L):
        got_k = conv(store.gpu.k_pages[torch.from_numpy(tables[layer]).to(DEV)].contiguous())
        got_v = conv(store.gpu.v_pages[torch.from_numpy(tables[layer]).to(DEV)].contiguous())
        assert np.array_equal(got_k, g["loaded_k"][layer])
        assert np.array_equal(got_v, g["loaded_v"][layer])


def _rand_kv(store: KVStore, seed: int):
    cfg = store.config
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(cfg.n_layers, cfg.n_kv_heads, cfg.head_dim, generator=g)
    v = torch.randn(cfg.n_layers, cfg.n_kv_heads, cfg.head_dim, generator=g)
    return k.to(DEV), v.to(DEV)


def test_reference_store_scenarios_on_cuda() -> None:
    # plastic-infer tests/test_kv_store.py scenarios, through this package on a CUDA pool.
    store = _store(torch.float32)
    cache = store.new_request()
    k, v = _rand_kv(store, 42)
    cache.append_token(k, v)
    phys = cache.block_table.get_page(0, 0)
    assert torch.equal(store.gpu.k_pages[phys, :, :, 0], k[0])
    assert torch.equal(store.gpu.v_pages[phys, :, :, 0], v[0])
    for i in range(4):
        cache.append_token(*_rand_kv(store, i))
    assert cache.block_table.num_logical_pages(0) == 2 and store.gpu.allocator.used_pages == 4
    # incremental sinking: 1.5 chunks -> 1 sunk; finishing the second -> 1 more
    store2 = _store(torch.float32)
    c = store2.new_request()
    toks: list[int] = []
    for i in range(12):
        c.append_token(*_rand_kv(store2, i))
        toks.append(i)
    c.set_token_ids(toks)
    assert store2.sink_completed_chunks(c) == 1 and store2.host_cache_size == 1
    for i in range(12, 16):
        c.append_token(*_rand_kv(store2, i))
        toks.append(i)
    c.set_token_ids(toks)
    assert store2.sink_completed_chunks(c) == 1 and store2.host_cache_size == 2
    # host LRU bound: 11 chunks into an 8-chunk host store
    store3 = _store(torch.float32)
    c3 = store3.new_request()
    for i in range(88):
        c3.append_token(*_rand_kv(store3, i * 11))
    c3.set_token_ids(list(range(88)))
    assert store3.sink_completed_chunks(c3) == 11
    assert store3.host_cache_size == 8
    # the surviving chunks are the 8 newest and hold the right data
    kept = [key for key in c3.chunk_keys if key.full_key in store3._host_cache]
    assert kept == c3.chunk_keys[3:]
    for ci, key in enumerate(c3.chunk_keys[3:], start=3):
        hk, _ = store3._host_cache[key.full_key]
        for t in range(8):
            pos = ci * 8 + t
            p = c3.block_table.get_page(1, pos // 4)
            assert torch.equal(hk[1, :, :, t], store3.gpu.k_pages[p, :, :, pos % 4].cpu())


def test_prefix_partial_hit_and_no_hit_on_cuda() -> None:
    store = _store(torch.float32)
    c1 = store.new_request()
    for i in range(8):
        c1.append_token(*_rand_kv(store, i))
    c1.set_token_ids(list(range(8)))
    store.sink_completed_chunks(c1)
    store.free_request(c1)
    c2 = store.new_request()
    matched, keys = store.load_prefix(c2, list(range(24)))
    assert matched == 8 and len(keys) == 1
    c3 = store.new_request()
    assert store.load_prefix(c3, [999, 998, 997]) == (0, [])
    assert c3.length == 0
