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

import numpy as np
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


def host_chunk_span_row(k: torch.Tensor, v: torch.Tensor) -> tuple[int, int, int, int, int, int]:
    """Span-table row of a host chunk at layer 0, from its K/V logical [L, H_kv, D, T] views
    over physical [L, H_kv, T, D] buffers: (K address, V address, T, and the element strides
    of the [H_kv, T, D] span: head, token, dim). Layer l's row adds l * H_kv * T * D *
    element size to both addresses."""
    L, H, D, T = k.shape
    want = (H * T * D, T * D, 1, D)
    if tuple(k.stride()) != want or tuple(v.stride()) != want or v.shape != k.shape:
        raise RuntimeError(f"unexpected host chunk layout {tuple(k.stride())}")
    return (k.data_ptr(), v.data_ptr(), T, T * D, D, 1)


class HostStoreDecoder:
    """Decode steps for requests whose KV outgrows the device pool (the host KV store
    wired into the decode loop).

    The reference keeps the host store's primitives (sink_completed_chunks, load_prefix,
    evict_chunks, host_stream_attention_v1; src/plastic_infer/kv/kv_store.py:230-386,
    src/plastic_infer/exec/attention.py:193-250) but its engine never calls them
    (src/plastic_infer/runtime/engine.py:501-539). This driver does, once per step:

    begin_step   every request gets the slot of its new token; when the pool has too few
                 free pages for them, the oldest host-backed chunks are evicted first.
    attend       per layer: the new K/V rows are written (one index-copy launch), the
                 requests that still hold all their chunks on the device are attended in
                 one paged_decode_attention launch, and every request with evicted chunks
                 by host-stream attention (host_stream_attention_v1's kernel) over its host
                 chunks (pinned, read in place) and its device tail. A host chunk's span
                 rows are built once, when it is first streamed, and a layer offsets them:
                 per call the host work is a few array operations, not per-chunk checks.
    end_step     completed chunks are sunk to the host store on the store's side stream
                 without waiting (KVStore.sink_completed_chunks_async), so the copies run
                 under the next step's attention, and chunks are evicted until the pool
                 holds at most `budget_pages` pages.

    Only chunks whose sink has been queued are evicted; each request keeps at least its
    newest complete chunk and its partial tail on the device (evict_chunks' rule).
    Inputs per layer are the step's post-RoPE q [B, Hq, D] and new k, v [B, Hkv, D].
    """

    def __init__(self, store: KVStore, caches: list[KVRequestCache],
                 budget_pages: int | None = None) -> None:
        self.store = store
        self.caches = caches
        cfg = store.config
        self.budget = store.gpu.total_pages if budget_pages is None else int(budget_pages)
        self.chunk_pages = cfg.n_layers * cfg.pages_per_chunk
        self.tables = BatchTables(store, caches)
        self.device = store.gpu.device
        self.workspace = kernels.default_workspace(self.device)
        self.positions: list[int] = []
        self.slots: torch.Tensor | None = None
        self.ctx_resident: torch.Tensor | None = None
        self.streamed: list[int] = []
        self.evictions = 0
        # per request: span-table rows (K address, V address, length, strides) of its
        # evicted host chunks at layer 0, oldest first; a layer adds layer * _layer_bytes
        # to both addresses (the chunk buffers are [L, H_kv, T, D])
        self._host_rows = [np.empty((0, 6), dtype=np.uint64) for _ in caches]
        elem = torch.tensor([], dtype=cfg.dtype).element_size()
        self._layer_bytes = cfg.n_kv_heads * cfg.tokens_per_chunk * cfg.head_dim * elem

    # -- pool budget -------------------------------------------------------------

    def used_pages(self) -> int:
        gpu = self.store.gpu
        return gpu.total_pages - gpu.allocator.free_pages

    def _evictable(self, cache: KVRequestCache) -> bool:
        c = cache.evicted_chunks
        return (c < cache.num_complete_chunks() - 1 and c < len(cache.chunk_keys)
                and self.store.has_host_chunk(cache.chunk_keys[c].full_key))

    def evict_to(self, max_used: int) -> int:
        """Evict one chunk at a time, from the request with the most resident complete
        chunks, until at most `max_used` pages are in use; returns pages freed."""
        freed = 0
        while self.used_pages() > max_used:
            cands = [c for c in self.caches if self._evictable(c)]
            if not cands:
                break
            victim = max(cands, key=lambda c: c.num_complete_chunks() - c.evicted_chunks)
            got = self.store.evict_chunks(self.chunk_pages, protected_request=victim)
            if got == 0:
                break
            freed += got
            self.evictions += 1
        return freed

    # -- one step ---------------------------------------------------------------

    def begin_step(self, token_ids: list[int] | None = None) -> None:
        """Reserve every request's next slot; `token_ids` (one per request) extend the
        requests' chunk keys, so the chunks they complete can be sunk."""
        cfg = self.store.config
        need = sum(cfg.n_layers for c in self.caches
                   if c.length % cfg.page_size == 0)  # a new page in every layer
        gpu = self.store.gpu
        if gpu.allocator.free_pages < need:
            self.evict_to(gpu.total_pages - need)
        self.positions = [c.length for c in self.caches]
        for i, c in enumerate(self.caches):
            c.reserve_tokens(1)
            if token_ids is not None:
                c.extend_token_ids([token_ids[i]])
        self.tables.refresh()
        L = cfg.n_layers
        self.slots = torch.tensor([[c.block_table.slot(l, p) for c, p in zip(self.caches, self.positions)]
                                   for l in range(L)], dtype=torch.int64, device=self.device)
        self.streamed = [b for b, c in enumerate(self.caches) if c.evicted_chunks > 0]
        for b in self.streamed:
            self._extend_host_rows(b)
        ctx = [0 if b in self.streamed else p + 1 for b, p in enumerate(self.positions)]
        self.ctx_resident = torch.tensor(ctx, dtype=torch.int32, device=self.device)

    def _extend_host_rows(self, b: int) -> None:
        """Add the span rows of request b's newly evicted chunks (checked once here: page-
        locked, [L, H_kv, T, D] buffers), after making the current stream wait for their
        sinks' copies."""
        cache = self.caches[b]
        rows = self._host_rows[b]
        n = cache.evicted_chunks
        if rows.shape[0] > n:  # evictions are only ever appended; rebuild if that changed
            rows = np.empty((0, 6), dtype=np.uint64)
        if rows.shape[0] == n:
            self._host_rows[b] = rows
            return
        stream = torch.cuda.current_stream(self.device)
        new = []
        for ci in range(rows.shape[0], n):
            k, v, ready = self.store.host_chunk(cache.chunk_keys[ci].full_key)
            if not (k.is_pinned() and v.is_pinned()):
                raise RuntimeError("host chunks must be page-locked to be read in place")
            if ready is not None:
                stream.wait_event(ready)  # the kernel reads the buffer after its sink's copy
            new.append(host_chunk_span_row(k, v))
        self._host_rows[b] = np.concatenate([rows, np.array(new, dtype=np.uint64)])

    def attend(self, layer: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
               out: torch.Tensor | None = None) -> torch.Tensor:
        gpu = self.store.gpu
        cfg = self.store.config
        kernels.kv_index_copy(gpu.k_phys, gpu.v_phys, k_new, v_new, self.slots[layer])
        # streamed requests get ctx 0 here (zeros), then their host-stream result
        out = kernels.paged_decode_attention(q, gpu.k_phys, gpu.v_phys, self.tables.tables[layer],
                                             self.ctx_resident, out=out, workspace=self.workspace)
        B, Hq, D = q.shape
        offset = np.uint64(layer * self._layer_bytes)
        for b in self.streamed:
            cache = self.caches[b]
            rows = self._host_rows[b]
            n = rows.shape[0]
            # the device tail: tokens after the evicted chunks, gathered from the pool
            start = cache.evicted_chunks * cfg.pages_per_chunk
            n_tail = cache.length - cache.evicted_chunks * cfg.tokens_per_chunk
            table = np.empty((n + (1 if n_tail > 0 else 0), 6), dtype=np.uint64)
            table[:n] = rows
            table[:n, :2] += offset
            if n_tail > 0:
                bt = self.tables.tables[layer, b, start:]
                rk = kernels.paged_kv_gather(gpu.k_phys, bt, n_tail)  # [R, H_kv, D]
                rv = kernels.paged_kv_gather(gpu.v_phys, bt, n_tail)
                table[n] = (rk.data_ptr(), rv.data_ptr(), n_tail, rk.stride(1), rk.stride(0),
                            rk.stride(2))
            kernels.host_stream_attention_table(q[b].view(1, Hq, D), out[b].view(1, Hq, D), table,
                                                cfg.n_kv_heads, q_start=self.positions[b],
                                                causal=True)
        return out

    def end_step(self) -> None:
        for c in self.caches:
            self.store.sink_completed_chunks_async(c)
        self.evict_to(self.budget)

    def step(self, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
             token_ids: list[int] | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
        """The KV path of one whole step: q [L, B, Hq, D], k_new/v_new [L, B, Hkv, D]."""
        self.begin_step(token_ids)
        if out is None:
            out = torch.empty_like(q)
        for layer in range(q.shape[0]):
            self.attend(layer, q[layer], k_new[layer], v_new[layer], out=out[layer])
        self.end_step()
        return out
