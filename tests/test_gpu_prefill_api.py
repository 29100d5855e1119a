"""Prefill through the reference-named API on a real KVStore (rows a2 / f3).

`exec.attention.paged_attention_v1` with several query tokens (SDPA's top-left causal or
non-causal) and `exec.runner_paged._attn_paged` with q_start_pos > 0 (the reference's
offset mask) run the tcgen05 paged prefill kernel straight from the pool when it covers
the shape, and the reference algorithm over the kernel gather otherwise (fp32 pools here).
Both are compared with the oracle at the attention tolerance (max-abs 2e-2 + rel 1e-2 for
bf16/f16, 1e-4 for fp32) on exactly the values stored in the pool.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import paged_kv_oracle as orc
from plastic_infer_b200.exec.attention import paged_attention_v1
from plastic_infer_b200.exec.runner_paged import _attn_paged, _write_kv_layer
from plastic_infer_b200.kv.kv_store import KVConfig, KVStore
from tests._helpers import assert_close, logical_f32

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)

CASES = [
    # (q_len, kv_len, q_start, causal, Hq, Hkv, D, S, dtype)
    (700, 700, 0, True, 32, 8, 128, 16, torch.bfloat16),     # first prefill
    (256, 1100, 844, True, 32, 8, 128, 16, torch.bfloat16),  # chunk at an offset
    (100, 333, 0, False, 32, 4, 128, 32, torch.float16),     # non-causal, G = 8
    (65, 200, 135, True, 8, 8, 64, 16, torch.bfloat16),      # MHA, head_dim 64
    (40, 90, 50, True, 4, 2, 64, 16, torch.float32),         # fp32: reference algorithm
]


@pytest.mark.parametrize("q_len,kv_len,q_start,causal,Hq,Hkv,D,S,dtype", CASES)
def test_prefill_through_the_reference_api(q_len, kv_len, q_start, causal, Hq, Hkv, D, S,
                                           dtype) -> None:
    cfg = KVConfig(n_layers=1, n_kv_heads=Hkv, head_dim=D, page_size=S,
                   max_pages=-(-kv_len // S) + 8, dtype=dtype, device=DEV)
    store = KVStore(cfg)
    cache = store.new_request()
    cache.reserve_tokens(kv_len)
    g = torch.Generator(device=DEV).manual_seed(kv_len + q_len)
    k = torch.randn((1, kv_len, Hkv, D), device=DEV, generator=g).to(dtype)
    v = torch.randn((1, kv_len, Hkv, D), device=DEV, generator=g).to(dtype)
    _write_kv_layer(cache, store, 0, 0, k, v)
    q = torch.randn((1, q_len, Hq, D), device=DEV, generator=g).to(dtype)
    table = cache.get_block_table_for_layer(0)
    if q_start == 0 or not causal:
        out = paged_attention_v1(q, store.gpu.k_pages, store.gpu.v_pages, table, S,
                                 kv_num_tokens=kv_len, causal=causal)
    else:
        out = _attn_paged(q, cache, 0, store, kv_num_tokens=kv_len, causal=True,
                          q_start_pos=q_start)
    torch.cuda.synchronize()
    ref = orc.paged_attention_prefill(q[0].float().cpu().numpy(), logical_f32(store.gpu.k_phys),
                                      logical_f32(store.gpu.v_phys), table, kv_len, q_start,
                                      causal, S)
    tol = (1e-4, 1e-4) if dtype == torch.float32 else (2e-2, 1e-2)
    assert out.shape == (1, q_len, Hq, D)
    assert_close(out[0].float().cpu().numpy(), ref, *tol)
