"""Host-side logic of the drop-in API, checked on CPU against the reference's behaviour.

Allocator traces and chunk keys are pinned by golden files produced by the
reference (tests/golden/allocator.json, chunk_keys.json). The store's bookkeeping
(page reservation, free, eviction, host LRU) runs on a CPU-device pool; data moves
on such a pool must raise (no CPU path).
"""

from __future__ import annotations

import json
import pathlib

import pytest
import torch

from plastic_infer_b200.kv import (BlockTable, KVConfig, KVStore, PageAllocator,
                                   compute_prefix_hashes, longest_prefix_hits)
from plastic_infer_b200.kv.chunk import compute_prefix_hashes_and_final

GOLD = pathlib.Path(__file__).resolve().parent / "golden"


def test_allocator_trace_matches_reference() -> None:
    trace = json.loads((GOLD / "allocator.json").read_text())
    a = PageAllocator(10)
    for step in trace:
        op = step["op"]
        if op[0] == "alloc":
            r = a.alloc()
        elif op[0] == "alloc_many":
            r = a.alloc_many(op[1])
        elif op[0] == "free":
            r = a.free(op[1])
        else:
            r = a.free_many(op[1])
        assert r == step["result"], step
        assert (a.free_pages, a.used_pages) == (step["free"], step["used"]), step


def test_allocator_errors_match_reference() -> None:
    a = PageAllocator(3)
    for _ in range(3):
        a.alloc()
    with pytest.raises(IndexError):
        a.alloc()
    with pytest.raises(IndexError):
        PageAllocator(5).alloc_many(10)
    b = PageAllocator(4)
    with pytest.raises(AssertionError):
        b.free(2)  # double free / never allocated
    with pytest.raises(AssertionError):
        PageAllocator(0)


def test_allocator_no_leak_random() -> None:
    # tests/test_paged.py:89-107 of the reference: seeded alloc/free never leaks.
    import random

    rng = random.Random(0)
    a = PageAllocator(64)
    live: list[int] = []
    for _ in range(2000):
        if live and (rng.random() < 0.5 or a.free_pages == 0):
            a.free(live.pop(rng.randrange(len(live))))
        else:
            live.append(a.alloc())
        assert a.used_pages == len(live)
        assert len(set(live)) == len(live)


def test_block_table_slots() -> None:
    bt = BlockTable(n_layers=2, page_size=4)
    for pid in (7, 2, 9):
        bt.append_page(0, pid)
    bt.append_page(1, 5)
    assert bt.slot(0, 0) == 28 and bt.slot(0, 5) == 9 and bt.slot(0, 11) == 39
    assert bt.slots_for(0, 3, 3) == [31, 8, 9]
    assert bt.chunk_page_ids(0, 2) == [7, 2, 5]
    assert bt.is_chunk_complete(0, 1) and not bt.is_chunk_complete(1, 1)
    assert bt.all_page_ids() == {2, 5, 7, 9}


def test_chunk_keys_match_reference() -> None:
    gold = json.loads((GOLD / "chunk_keys.json").read_text())
    for name, case in gold.items():
        keys = compute_prefix_hashes(case["tokens"], chunk_size=case["chunk_size"])
        assert [k.prefix_key.hex() for k in keys] == case["prefix"], name
        assert [k.cumulative_key.hex() for k in keys] == case["cumulative"], name
    with pytest.raises(ValueError):
        compute_prefix_hashes(list(range(5)), chunk_size=4)


def test_longest_prefix_hits() -> None:
    toks = list(range(40))
    keys, _ = compute_prefix_hashes_and_final(toks[:32], chunk_size=8)
    index = {k.full_key: k for k in keys[:3]}
    matched, tail = longest_prefix_hits(index, toks, chunk_size=8)
    assert len(matched) == 3 and tail == 24
    other = toks[:8] + [999] * 8 + toks[16:]
    matched, tail = longest_prefix_hits(index, other, chunk_size=8)
    assert len(matched) == 1 and tail == 8
    assert longest_prefix_hits({}, toks, chunk_size=8) == ([], 0)


def _cpu_store(**kw) -> KVStore:
    cfg = dict(n_layers=2, n_kv_heads=2, head_dim=4, page_size=4, pages_per_chunk=2,
               max_pages=64, max_host_chunks=8, dtype=torch.float32, device=torch.device("cpu"))
    cfg.update(kw)
    return KVStore(KVConfig(**cfg))


def test_store_bookkeeping_on_cpu_pool() -> None:
    store = _cpu_store()
    assert store.config.bytes_per_page == 2 * 4 * 4 * 2 * 4
    assert store.config.tokens_per_chunk == 8
    # logical views keep the reference's shape
    assert store.gpu.k_pages.shape == (64, 2, 4, 4)
    assert store.gpu.get_page_k(3).shape == (2, 4, 4)
    cache = store.new_request()
    cache.reserve_tokens(5)   # 5 tokens -> 2 pages per layer
    assert cache.length == 5
    assert cache.block_table.num_logical_pages(0) == 2
    assert store.gpu.allocator.used_pages == 4
    # reference page order: layer 0 and 1 alternate per new page
    assert cache.get_block_table_for_layer(0) == [0, 2]
    assert cache.get_block_table_for_layer(1) == [1, 3]
    store.free_request(cache)
    assert store.gpu.allocator.used_pages == 0


def test_store_eviction_policy_matches_reference() -> None:
    # tests/test_kv_store.py:268-284 of the reference, on the bookkeeping only.
    store = _cpu_store()
    cache = store.new_request()
    cache.reserve_tokens(8 * 4)           # 4 full chunks
    cache.set_token_ids(list(range(32)))
    assert cache.num_complete_chunks() == 4 and len(cache.chunk_keys) == 4
    used = store.gpu.allocator.used_pages
    freed = store.evict_chunks(need_pages=1, protected_request=cache)
    assert freed == 4                      # one chunk = 2 layers x 2 pages
    assert store.gpu.allocator.used_pages == used - freed
    assert store.evict_chunks(need_pages=1) == 0  # no protected request -> no-op
    # The reference leaves the freed pages in the block table (kv_store.py:380-383), so
    # its second eviction walks chunk 0 again and trips the allocator's double-free
    # assertion ("page 0 not in use"). Fixed: the evicted entries are -1 and the next
    # call continues with chunk 1; the newest complete chunk (3) is still kept.
    assert cache.evicted_chunks == 1
    assert cache.get_block_table_for_layer(0)[:2] == [-1, -1]
    assert cache.get_block_table_for_layer(1)[:2] == [-1, -1]
    assert store.evict_chunks(need_pages=100, protected_request=cache) == 8
    assert cache.evicted_chunks == 3
    assert store.gpu.allocator.used_pages == used - 12
    assert store.evict_chunks(need_pages=100, protected_request=cache) == 0
    assert all(p >= 0 for p in cache.get_block_table_for_layer(0)[6:])
    store.free_request(cache)              # frees only the pages still held
    assert store.gpu.allocator.used_pages == 0


def test_evicted_chunk_host_copies_are_held_while_the_request_lives() -> None:
    # evicted chunks' host copies are the only copy left: the host LRU must skip them
    store = _cpu_store()
    cache = store.new_request()
    cache.reserve_tokens(8 * 3)
    cache.set_token_ids(list(range(24)))
    k0 = cache.chunk_keys[0].full_key
    store._host_cache[k0] = (None, None)  # as if sunk (the data move itself needs a GPU)
    store._touch_host(k0)
    store.evict_chunks(need_pages=1, protected_request=cache)
    assert store._host_pins == {k0: 1}
    assert store._evict_host_lru() is False    # the only cached chunk is held
    assert k0 in store._host_cache
    store.free_request(cache)
    assert store._host_pins == {}
    assert store._evict_host_lru() is True
    assert k0 not in store._host_cache


def test_data_moves_need_cuda() -> None:
    store = _cpu_store()
    cache = store.new_request()
    k = torch.zeros(2, 2, 4)
    with pytest.raises((ValueError, RuntimeError)):
        cache.append_token(k, k)
    cache.reserve_tokens(8)
    cache.set_token_ids(list(range(8)))
    with pytest.raises(RuntimeError):
        store.sink_completed_chunks(cache)


def test_streaming_an_unsunk_evicted_chunk_raises() -> None:
    # the reference frees a chunk whether or not it was sunk; its K/V are then gone, and
    # attending the request from the host store must say so instead of reading nothing
    store = _cpu_store()
    cache = store.new_request()
    cache.reserve_tokens(8 * 3)
    cache.set_token_ids(list(range(24)))
    assert store.evict_chunks(need_pages=1, protected_request=cache) == 4
    with pytest.raises(RuntimeError, match="without a host copy"):
        store.host_stream_chunks(cache, 0)


def test_extend_token_ids_gives_the_keys_of_set_token_ids() -> None:
    import numpy as np
    import torch

    from plastic_infer_b200.kv.kv_store import KVConfig, KVStore

    cfg = KVConfig(n_layers=1, n_kv_heads=1, head_dim=8, page_size=4, pages_per_chunk=2,
                   max_pages=8, device=torch.device("cpu"))
    store = KVStore(cfg)
    rng = np.random.default_rng(0)
    ids = [int(x) for x in rng.integers(0, 2**32 - 1, 61, dtype=np.uint64)]
    whole = store.new_request(0)
    whole.set_token_ids(ids)
    step = store.new_request(1)
    step.set_token_ids(ids[:5])
    cur, added = 5, 0
    for n in (1, 2, 9, 1, 20, 23):
        added += step.extend_token_ids(ids[cur:cur + n])
        cur += n
    assert cur == len(ids)
    assert added == len(whole.chunk_keys) == 7
    assert step.chunk_keys == whole.chunk_keys
    assert step._final_hash == whole._final_hash


def test_host_chunk_span_rows_match_the_generic_span_path() -> None:
    # HostStoreDecoder keeps one row per host chunk (layer 0) and offsets it by the layer;
    # that must equal the row host_stream_attention builds from the chunk's layer view
    # (kv[layer] of the logical [L, H, D, T] view, permuted to [H, T, D]).
    import numpy as np

    from plastic_infer_b200.decode import host_chunk_span_row

    L, H, T, D = 5, 3, 32, 16
    for dtype in (torch.bfloat16, torch.float32):
        kp = torch.zeros((L, H, T, D), dtype=dtype)
        vp = torch.zeros_like(kp)
        k, v = kp.permute(0, 1, 3, 2), vp.permute(0, 1, 3, 2)   # the store's logical views
        row = np.array(host_chunk_span_row(k, v), dtype=np.uint64)
        layer_bytes = H * T * D * kp.element_size()
        for layer in range(L):
            ks, vs = k[layer].permute(0, 2, 1), v[layer].permute(0, 2, 1)
            want = (ks.data_ptr(), vs.data_ptr(), ks.shape[1], ks.stride(0), ks.stride(1),
                    ks.stride(2))
            got = row.copy()
            got[:2] += np.uint64(layer * layer_bytes)
            assert tuple(int(x) for x in got) == want
    with pytest.raises(RuntimeError):
        bad = torch.zeros((L, H, D, T))  # contiguous logical layout: not the store's buffers
        host_chunk_span_row(bad, bad)
