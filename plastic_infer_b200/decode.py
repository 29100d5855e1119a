"""Batched decode over the paged pool: many requests, one launch per kernel per layer.

The reference decodes one request at a time: every layer of every request turns its
block table from a Python list into a tensor (src/plastic_infer/exec/attention.py:134),
gathers the whole context and runs SDPA (src/plastic_infer/exec/runner_paged.py:235-269,
called per request by src/plastic_infer/runtime/engine.py:530-536). Here a step of B
requests keeps device-resident block tables [n_layers, B, max_pages] (int32), context
lengths [B] and slot mappings [n_layers, B], refreshed only when the host allocator
hands out a page. Past the projections, each layer costs two launches for the whole
batch: `decode_prologue` (QK-norm, RoPE, and the write of the new K/V rows) and
`paged_decode_attention`.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import kernels
from .exec.attention import rms_norm
from .exec.runner import DenseWeights, ModelConfig, linear
from .kv.kv_store import KVRequestCache, KVStore


class BatchTables:
    """Device mirror of a batch's block tables, lengths and next-token slots."""

    def __init__(self, store: KVStore, caches: list[KVRequestCache], grow: int = 64) -> None:
        self.store = store
        self.caches = caches
        self.grow = grow
        self.device = store.gpu.device
        self.width = 0
        self.tables: torch.Tensor | None = None      # [L, B, width] int32
        self._host_pages = [[0] * store.config.n_layers for _ in caches]

    def refresh(self) -> None:
        """Copy rows whose page lists grew since the last refresh."""
        cfg = self.store.config
        L, B = cfg.n_layers, len(self.caches)
        need = max((c.block_table.num_logical_pages(l) for c in self.caches for l in range(L)), default=0)
        if self.tables is None or need > self.width:
            self.width = max(need + self.grow, 1)
            full = torch.zeros((L, B, self.width), dtype=torch.int32)
            for b, c in enumerate(self.caches):
                for l in range(L):
                    row = c.block_table.pages[l]
                    full[l, b, :len(row)] = torch.tensor(row, dtype=torch.int32)
                    self._host_pages[b][l] = len(row)
            self.tables = full.to(self.device)
            return
        for b, c in enumerate(self.caches):
            for l in range(L):
                row = c.block_table.pages[l]
                have = self._host_pages[b][l]
                if len(row) > have:
                    self.tables[l, b, have:len(row)] = torch.tensor(row[have:], dtype=torch.int32,
                                                                    device=self.device)
                    self._host_pages[b][l] = len(row)


def decode_step_paged_batched(weights: DenseWeights, config: ModelConfig, store: KVStore,
                              caches: list[KVRequestCache], input_ids: list[int],
                              tables: BatchTables | None = None) -> torch.Tensor:
    """One greedy-decode step for B requests; returns logits [B, vocab].

    Per request the math is decode_step_paged's (src/plastic_infer/exec/runner_paged.py:209-274),
    with the QK-norm of the MoE runner when the config has it
    (src/plastic_infer/exec/runner_moe_paged.py:135-142); requests may have different
    lengths. RoPE angles are pos * inv_freq in fp32, the values of the reference's fp32
    table; the reference builds its table in the model dtype, which in bf16 runs rounds
    the angles of late positions.
    """
    B = len(caches)
    dev, dt = weights.device, weights.dtype
    cfg = config
    positions = [c.length for c in caches]
    for c in caches:
        c.reserve_tokens(1)
    if tables is None:
        tables = BatchTables(store, caches)
    tables.refresh()
    L = cfg.n_layers
    slots = torch.tensor([[c.block_table.slot(l, p) for c, p in zip(caches, positions)]
                          for l in range(L)], dtype=torch.int64, device=dev)
    ctx = torch.tensor([p + 1 for p in positions], dtype=torch.int32, device=dev)
    pos_t = torch.tensor(positions, dtype=torch.int64, device=dev)
    inv_freq = kernels.rope_inv_freq(cfg.head_dim, float(cfg.rope_base), dev)
    x = weights["embed_tokens.weight"][torch.tensor(input_ids, device=dev)].to(dt).view(B, 1, -1)
    gpu = store.gpu
    for l in range(L):
        p = f"layers.{l}."
        h = rms_norm(x, weights[p + "input_layernorm.weight"])
        q = linear(h, weights[p + "self_attn.q_proj.weight"]).view(B, cfg.n_heads, cfg.head_dim)
        k = linear(h, weights[p + "self_attn.k_proj.weight"]).view(B, cfg.n_kv_heads, cfg.head_dim)
        v = linear(h, weights[p + "self_attn.v_proj.weight"]).view(B, cfg.n_kv_heads, cfg.head_dim)
        qw = kw = None
        if cfg.qk_norm:
            qw, kw = weights[p + "self_attn.q_norm.weight"], weights[p + "self_attn.k_norm.weight"]
        # one launch: QK-norm + RoPE of q and k, new K/V rows written at their slots
        qr = kernels.decode_prologue(q, k, v, pos_t, inv_freq, slots[l], gpu.k_phys, gpu.v_phys,
                                     qw, kw)
        attn = kernels.paged_decode_attention(qr, gpu.k_phys, gpu.v_phys, tables.tables[l], ctx)
        attn = attn.to(dt).view(B, 1, cfg.n_heads * cfg.head_dim)
        x = x + linear(attn, weights[p + "self_attn.o_proj.weight"])
        h = rms_norm(x, weights[p + "post_attention_layernorm.weight"])
        ffn = F.silu(linear(h, weights[p + "mlp.gate_proj.weight"])) * linear(h, weights[p + "mlp.up_proj.weight"])
        x = x + linear(ffn, weights[p + "mlp.down_proj.weight"])
    x = rms_norm(x, weights["norm.weight"])
    return linear(x[:, -1, :], weights["lm_head.weight"])
