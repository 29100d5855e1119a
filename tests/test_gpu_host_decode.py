"""GPU parity of the host-store decode driver (decode.HostStoreDecoder).

Three requests decode past a device pool budget smaller than their KV. Each step the
driver writes the new rows, attends resident requests with the paged kernel and
requests with evicted chunks through host-stream attention (host chunks read in place
plus the device tail), sinks completed chunks without waiting and evicts down to the
budget. Every step's outputs are compared with the oracle over each request's full
token history (the K/V it was given, kept here on the host), at the attention
tolerance (max-abs 2e-2 + rel 1e-2 of the fp32 path on the same bf16 inputs); the host
chunks must hold the original rows bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import paged_kv_oracle as orc
from plastic_infer_b200 import kernels
from plastic_infer_b200.decode import HostStoreDecoder
from plastic_infer_b200.kv.kv_store import KVConfig, KVStore
from tests._helpers import assert_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
ATOL, RTOL = 2e-2, 1e-2


def _ref_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, S: int) -> np.ndarray:
    """Oracle attention of q [Hq, D] over K/V rows [T, Hkv, D] (one request)."""
    T, H, D = k.shape
    npg = -(-T // S)
    pad = np.zeros((npg * S - T, H, D), np.float32)
    kp = np.concatenate([k, pad]).reshape(npg, S, H, D).transpose(0, 2, 3, 1)
    vp = np.concatenate([v, pad]).reshape(npg, S, H, D).transpose(0, 2, 3, 1)
    return orc.paged_attention_decode(q[None], kp, vp, [list(range(npg))], [T], S)[0]


def _bf16(rng: np.random.Generator, shape) -> torch.Tensor:
    return torch.from_numpy(rng.standard_normal(shape, dtype=np.float32)).to(torch.bfloat16)


@pytest.mark.parametrize("budget", [24, 40])
def test_host_store_decoder_matches_oracle_past_the_pool(budget: int) -> None:
    L, Hkv, Hq, D, S, ppc = 2, 2, 8, 64, 16, 2        # 32-token chunks
    cfg = KVConfig(n_layers=L, n_kv_heads=Hkv, head_dim=D, page_size=S, pages_per_chunk=ppc,
                   max_pages=48, max_host_chunks=64, dtype=torch.bfloat16, device=DEV)
    store = KVStore(cfg)
    rng = np.random.default_rng(budget)
    prompts = [90, 64, 33]
    caches, truth_k, truth_v, tokens = [], [], [], []
    for i, n in enumerate(prompts):
        c = store.new_request(request_id=i)
        c.reserve_tokens(n)
        k = _bf16(rng, (n, L, Hkv, D))
        v = _bf16(rng, (n, L, Hkv, D))
        slots = torch.tensor([c.block_table.slot(l, t) for t in range(n) for l in range(L)],
                             dtype=torch.int64, device=DEV)
        kernels.kv_index_copy(store.gpu.k_phys, store.gpu.v_phys,
                              k.reshape(n * L, Hkv, D).to(DEV), v.reshape(n * L, Hkv, D).to(DEV), slots)
        ids = [int(x) for x in rng.integers(0, 50000, n)]
        c.set_token_ids(ids)
        caches.append(c)
        truth_k.append([k.float().numpy()])
        truth_v.append([v.float().numpy()])
        tokens.append(ids)
    dec = HostStoreDecoder(store, caches, budget_pages=budget)
    for c in caches:
        store.sink_completed_chunks(c)
    dec.evict_to(budget)

    streamed_steps = 0
    for step in range(48):
        B = len(caches)
        q = _bf16(rng, (L, B, Hq, D)).to(DEV)
        kn = _bf16(rng, (L, B, Hkv, D))
        vn = _bf16(rng, (L, B, Hkv, D))
        new_ids = [int(x) for x in rng.integers(0, 50000, B)]
        out = dec.step(q, kn.to(DEV), vn.to(DEV), token_ids=new_ids)
        torch.cuda.synchronize()
        streamed_steps += bool(dec.streamed)
        got = out.float().cpu().numpy()
        for b in range(B):
            truth_k[b].append(kn[:, b].float().numpy()[None])   # [1, L, Hkv, D]
            truth_v[b].append(vn[:, b].float().numpy()[None])
            tokens[b].append(new_ids[b])
            K = np.concatenate(truth_k[b])
            V = np.concatenate(truth_v[b])
            for layer in range(L):
                ref = _ref_attention(q[layer, b].float().cpu().numpy(), K[:, layer], V[:, layer], S)
                assert_close(got[layer, b], ref, ATOL, RTOL)
    assert dec.evictions > 0 and streamed_steps > 0
    assert store.gpu.total_pages - store.gpu.allocator.free_pages <= budget + L * len(caches)

    # host chunks of evicted chunks hold the original rows, bit for bit
    torch.cuda.synchronize()
    tpc = S * ppc
    checked = 0
    for b, c in enumerate(caches):
        K = np.concatenate(truth_k[b])
        for ci in range(c.evicted_chunks):
            hk, _ = store._host_cache[c.chunk_keys[ci].full_key]      # [L, Hkv, D, tpc]
            want = K[ci * tpc:(ci + 1) * tpc].transpose(1, 2, 3, 0)   # [L, Hkv, D, tpc]
            assert np.array_equal(hk.float().numpy(), want)
            checked += 1
    assert checked > 0


def test_async_sink_orders_page_reuse_and_host_reads() -> None:
    # A chunk sunk without waiting, evicted at once, its pages handed to another request
    # and overwritten: attention over the first request's host copy still sees the
    # original rows (the store orders the reuse after the gather).
    L, Hkv, Hq, D, S, ppc = 2, 2, 4, 64, 16, 2
    cfg = KVConfig(n_layers=L, n_kv_heads=Hkv, head_dim=D, page_size=S, pages_per_chunk=ppc,
                   max_pages=16, max_host_chunks=8, dtype=torch.bfloat16, device=DEV)
    store = KVStore(cfg)
    rng = np.random.default_rng(5)
    a = store.new_request(0)
    n = 70                                           # two complete chunks + 6 tokens
    a.reserve_tokens(n)
    k = _bf16(rng, (n, L, Hkv, D))
    v = _bf16(rng, (n, L, Hkv, D))
    slots = torch.tensor([a.block_table.slot(l, t) for t in range(n) for l in range(L)],
                         dtype=torch.int64, device=DEV)
    kernels.kv_index_copy(store.gpu.k_phys, store.gpu.v_phys, k.reshape(-1, Hkv, D).to(DEV),
                          v.reshape(-1, Hkv, D).to(DEV), slots)
    a.set_token_ids([int(x) for x in rng.integers(0, 1000, n)])
    count, ev = store.sink_completed_chunks_async(a)
    assert count == 2 and ev is not None
    freed = store.evict_chunks(L * ppc, protected_request=a)     # chunk 0's pages
    assert freed == L * ppc and a.evicted_chunks == 1
    b = store.new_request(1)
    b.reserve_tokens(S * ppc)                                     # takes the freed pages
    junk = torch.full((S * ppc * L, Hkv, D), 7.0, dtype=torch.bfloat16, device=DEV)
    sb = torch.tensor([b.block_table.slot(l, t) for t in range(S * ppc) for l in range(L)],
                      dtype=torch.int64, device=DEV)
    kernels.kv_index_copy(store.gpu.k_phys, store.gpu.v_phys, junk, junk, sb)
    q = _bf16(rng, (1, 1, Hq, D)).to(DEV)
    from plastic_infer_b200.exec.attention import host_stream_attention_v1
    for layer in range(L):
        chunks, rk, rv = store.host_stream_chunks(a, layer)
        out = host_stream_attention_v1(q, chunks, rk, rv, q_start_pos=n - 1)
        ref = _ref_attention(q[0, 0].float().cpu().numpy(), k[:, layer].float().numpy(),
                             v[:, layer].float().numpy(), S)
        assert_close(out[0, 0].float().cpu().numpy(), ref, ATOL, RTOL)
