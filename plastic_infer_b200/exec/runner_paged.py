"""Dense model x paged KV runner, on the sm_100a KV path.

Drop-in for src/plastic_infer/exec/runner_paged.py: same functions and signatures.
The KV path is replaced:

* `_write_kv_layer` resolves the token range to flat slots on the host and writes
  all of them with one `kv_index_copy` launch (reference: 2 strided copies per token,
  runner_paged.py:123-129).
* `_allocate_pages_for_tokens` reserves pages without writing the zero rows the
  reference appends first (runner_paged.py:98-109): every reserved slot is written by
  `_write_kv_layer` before it is read.
* `_attn_paged` -> `paged_attention_v1`, which for a decode query is the paged decode
  kernel.

The model math around it (RMSNorm, projections, RoPE, SwiGLU) follows the reference
(runner_paged.py:132-274) so logits can be compared with the reference's.
"""

from __future__ import annotations

from functools import lru_cache

import torch
import torch.nn.functional as F

from .. import kernels
from ..kv.kv_store import KVConfig, KVRequestCache, KVStore
from .attention import (build_rope_cache, gather_paged_kv, paged_attention_v1, qk_norm, rms_norm,
                        rope_positions)
from .runner import DenseWeights, ModelConfig, linear


def make_kv_config(model_cfg: ModelConfig, max_pages: int = 256, max_host_chunks: int = 64,
                   device: torch.device | None = None,
                   dtype: torch.dtype | None = None) -> KVConfig:
    """KVConfig for a model (runner_paged.py:20-33)."""
    return KVConfig(
        n_layers=model_cfg.n_layers,
        n_kv_heads=model_cfg.n_kv_heads,
        head_dim=model_cfg.head_dim,
        max_pages=max_pages,
        max_host_chunks=max_host_chunks,
        dtype=dtype or model_cfg.dtype,
        device=device or torch.device("cpu"),
    )


def _attn_paged(q: torch.Tensor, cache: KVRequestCache, layer_idx: int, store: KVStore,
                kv_num_tokens: int | None = None, causal: bool = True,
                q_start_pos: int = 0) -> torch.Tensor:
    """Paged attention for one request and layer (runner_paged.py:36-95)."""
    cfg = store.config
    block_table = cache.get_block_table_for_layer(layer_idx)
    if not causal or q_start_pos == 0:
        return paged_attention_v1(q, store.gpu.k_pages, store.gpu.v_pages, block_table,
                                  cfg.page_size, kv_num_tokens=kv_num_tokens, causal=causal)
    # Incremental prefill: Q row i sits at position q_start_pos + i and sees
    # KV[0 : q_start_pos + i + 1] (runner_paged.py:61-95). The tcgen05 prefill kernel
    # applies that mask itself, reading the pages in place; shapes it does not cover keep
    # the reference's dense mask over the kernel gather.
    q_len = q.shape[1]
    kv_len = kv_num_tokens or (len(block_table) * cfg.page_size)
    kp = store.gpu.k_phys
    if kv_len > 0 and kernels.prefill_supported(q, kp):
        n_pages = -(-kv_len // cfg.page_size)
        bt = torch.tensor(block_table[:n_pages], dtype=torch.int32, device=kp.device)
        return kernels.paged_prefill_attention(q, kp, store.gpu.v_phys, bt, kv_len,
                                               q_start=q_start_pos, causal=True, impl="tc")
    dev = q.device
    q_pos = torch.arange(q_start_pos, q_start_pos + q_len, device=dev)
    kv_pos = torch.arange(kv_len, device=dev)
    mask = torch.zeros(q_len, kv_len, dtype=q.dtype, device=dev)
    mask = mask.masked_fill(kv_pos[None, :] > q_pos[:, None], float("-inf"))[None, None]
    k, v = gather_paged_kv(store.gpu.k_pages, store.gpu.v_pages, block_table, cfg.page_size,
                           kv_num_tokens)
    q_t, k_t, v_t = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    Hq, Hkv = q_t.shape[1], k_t.shape[1]
    if Hq != Hkv:
        k_t = k_t.repeat_interleave(Hq // Hkv, dim=1)
        v_t = v_t.repeat_interleave(Hq // Hkv, dim=1)
    return F.scaled_dot_product_attention(q_t, k_t, v_t, attn_mask=mask).transpose(1, 2)


def _allocate_pages_for_tokens(cache: KVRequestCache, store: KVStore, n_tokens: int) -> None:
    """Reserve pages for n_tokens new positions (runner_paged.py:98-109)."""
    cache.reserve_tokens(n_tokens)


def _write_kv_layer(cache: KVRequestCache, store: KVStore, layer_idx: int, start_pos: int,
                    k: torch.Tensor, v: torch.Tensor) -> None:
    """Write k, v [1, T, n_kv_heads, head_dim] at positions start_pos.. of one layer
    (runner_paged.py:112-129) with a single index-copy launch."""
    T = k.shape[1]
    if T == 0:
        return
    slots = cache.block_table.slots_for(layer_idx, start_pos, T)
    gpu = store.gpu
    slot_t = torch.tensor(slots, dtype=torch.int64, device=gpu.device)
    kernels.kv_index_copy(gpu.k_phys, gpu.v_phys, k[0].to(gpu.dtype), v[0].to(gpu.dtype), slot_t)


@lru_cache(maxsize=8)
def _rope_table(seq_len: int, head_dim: int, base: float, device: torch.device,
                dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    # The reference rebuilds this table every step (runner_paged.py:231-232); the
    # values depend only on the arguments, so it is built once.
    return build_rope_cache(seq_len, head_dim, base=base, device=device, dtype=dtype)


def _layer_qkv(weights: DenseWeights, cfg: ModelConfig, layer_idx: int, x: torch.Tensor,
               seq_len: int, cos: torch.Tensor, sin: torch.Tensor, positions: torch.Tensor):
    p = f"layers.{layer_idx}."
    h = rms_norm(x, weights[p + "input_layernorm.weight"])
    q = linear(h, weights[p + "self_attn.q_proj.weight"]).view(1, seq_len, cfg.n_heads, cfg.head_dim)
    k = linear(h, weights[p + "self_attn.k_proj.weight"]).view(1, seq_len, cfg.n_kv_heads, cfg.head_dim)
    v = linear(h, weights[p + "self_attn.v_proj.weight"]).view(1, seq_len, cfg.n_kv_heads, cfg.head_dim)
    if cfg.qk_norm:
        q, k = qk_norm(q, k, weights[p + "self_attn.q_norm.weight"],
                       weights[p + "self_attn.k_norm.weight"], cfg.head_dim)
    q = rope_positions(cos, sin, positions, q)
    k = rope_positions(cos, sin, positions, k)
    return q, k, v


def _layer_out(weights: DenseWeights, cfg: ModelConfig, layer_idx: int, residual: torch.Tensor,
               attn: torch.Tensor, seq_len: int) -> torch.Tensor:
    p = f"layers.{layer_idx}."
    attn = attn.contiguous().view(1, seq_len, cfg.n_heads * cfg.head_dim)
    x = residual + linear(attn, weights[p + "self_attn.o_proj.weight"])
    h = rms_norm(x, weights[p + "post_attention_layernorm.weight"])
    ffn = F.silu(linear(h, weights[p + "mlp.gate_proj.weight"])) * linear(h, weights[p + "mlp.up_proj.weight"])
    return x + linear(ffn, weights[p + "mlp.down_proj.weight"])


def prefill_forward_paged(weights: DenseWeights, config: ModelConfig, store: KVStore,
                          cache: KVRequestCache, input_ids: torch.Tensor,
                          start_pos: int = 0) -> torch.Tensor:
    """Prefill `input_ids` [seq_len] after `start_pos` cached tokens; returns the last
    token's logits [vocab] (runner_paged.py:132-206)."""
    assert input_ids.dim() == 1
    seq_len = input_ids.shape[0]
    dev, dt = weights.device, weights.dtype
    _allocate_pages_for_tokens(cache, store, seq_len)
    x = weights["embed_tokens.weight"][input_ids.to(dev)].to(dt).unsqueeze(0)
    cos, sin = _rope_table(config.max_seq_len, config.head_dim, float(config.rope_base), dev, dt)
    positions = torch.arange(start_pos, start_pos + seq_len, device=dev)
    for layer_idx in range(config.n_layers):
        q, k, v = _layer_qkv(weights, config, layer_idx, x, seq_len, cos, sin, positions)
        _write_kv_layer(cache, store, layer_idx, start_pos, k, v)
        attn = _attn_paged(q, cache, layer_idx, store, kv_num_tokens=start_pos + seq_len,
                           causal=True, q_start_pos=start_pos)
        x = _layer_out(weights, config, layer_idx, x, attn, seq_len)
    x = rms_norm(x, weights["norm.weight"])
    return linear(x[:, -1, :], weights["lm_head.weight"]).squeeze(0)


def decode_step_paged(weights: DenseWeights, config: ModelConfig, store: KVStore,
                      cache: KVRequestCache, input_id: int) -> torch.Tensor:
    """One decode step; returns logits [vocab] (runner_paged.py:209-274)."""
    dev, dt = weights.device, weights.dtype
    pos = cache.length
    _allocate_pages_for_tokens(cache, store, 1)
    x = weights["embed_tokens.weight"][input_id].to(dt).view(1, 1, -1)
    cos, sin = _rope_table(config.max_seq_len, config.head_dim, float(config.rope_base), dev, dt)
    pos_t = torch.tensor([pos], device=dev)
    for layer_idx in range(config.n_layers):
        q, k, v = _layer_qkv(weights, config, layer_idx, x, 1, cos, sin, pos_t)
        _write_kv_layer(cache, store, layer_idx, pos, k, v)
        attn = _attn_paged(q, cache, layer_idx, store, kv_num_tokens=pos + 1, causal=False)
        x = _layer_out(weights, config, layer_idx, x, attn, 1)
    x = rms_norm(x, weights["norm.weight"])
    return linear(x[:, -1, :], weights["lm_head.weight"]).squeeze(0)
