"""KV store on the B200 paged pool: device pages, per-request caches, host chunk store.

Drop-in for the reference's kv/kv_store.py (src/plastic_infer/kv/kv_store.py:46-406):
same classes, methods, arguments and error behaviour. What changes is underneath:

* Physical pool layout. `KVPagedStorage` stores K and V as
  [total_pages, n_kv_heads, page_size, head_dim] and exposes the reference's logical
  [total_pages, n_kv_heads, head_dim, page_size] as `k_pages` / `v_pages` views, so
  reference-style indexing (`k_pages[p, :, :, off] = ...`, `k_pages[p].to(...)`)
  still reads and writes the same elements. A (page, head) tile is one contiguous
  page_size*head_dim block: a TMA box for attention, a 256-byte row per token per
  head for the index-copy.
* KV writes. `append_token` writes all layers of a token with one
  `kv_index_copy` launch (reference: 2 strided copies per layer,
  kv_store.py:140-143).
* Host chunk store. Host chunks live in pinned memory, physically
  [n_layers, n_kv_heads, tokens_per_chunk, head_dim]; `_host_cache` values are the
  logical [n_layers, n_kv_heads, head_dim, tokens_per_chunk] views the reference
  exposes (kv_store.py:252-256). Sinking gathers every page of every new chunk
  into a device staging buffer with one `page_gather` launch and copies it to the
  host with one cudaMemcpyAsync per chunk on a side stream; `load_prefix` does the
  reverse with `page_scatter` (reference: one synchronous .to() per (layer, page),
  kv_store.py:258-269, 311-321).

Device pools on a non-CUDA device are allowed so host-side bookkeeping (allocator,
block tables, chunk keys, eviction) can be exercised anywhere, but every data move
raises there: there is no CPU path.
"""

from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Optional

import torch

from .. import kernels
from .chunk import (ChunkKey, compute_prefix_hashes_and_final, longest_prefix_hits,
                    next_chunk_key)
from .paged import DEFAULT_CHUNK_PAGES, DEFAULT_PAGE_SIZE, BlockTable, PageAllocator


@dataclass
class KVConfig:
    """Shape parameters for the KV store (src/plastic_infer/kv/kv_store.py:46-67)."""

    n_layers: int
    n_kv_heads: int
    head_dim: int
    page_size: int = DEFAULT_PAGE_SIZE
    pages_per_chunk: int = DEFAULT_CHUNK_PAGES
    max_pages: int = 1024
    max_host_chunks: int = 256
    dtype: torch.dtype = torch.float32
    device: torch.device = field(default_factory=lambda: torch.device("cpu"))

    @property
    def bytes_per_page(self) -> int:
        per_page = self.n_kv_heads * self.head_dim * self.page_size * 2
        return per_page * torch.tensor([], dtype=self.dtype).element_size()

    @property
    def tokens_per_chunk(self) -> int:
        return self.page_size * self.pages_per_chunk


class KVPagedStorage:
    """Physical page pool on one device (src/plastic_infer/kv/kv_store.py:70-95)."""

    def __init__(self, config: KVConfig, total_pages: int,
                 device: Optional[torch.device] = None,
                 dtype: Optional[torch.dtype] = None) -> None:
        self.config = config
        self.device = torch.device(device or config.device)
        self.dtype = dtype or config.dtype
        self.total_pages = total_pages
        self.allocator = PageAllocator(total_pages)
        shape = (total_pages, config.n_kv_heads, config.page_size, config.head_dim)
        self.k_phys = torch.zeros(shape, dtype=self.dtype, device=self.device)
        self.v_phys = torch.zeros(shape, dtype=self.dtype, device=self.device)

    @property
    def k_pages(self) -> torch.Tensor:
        """Logical [total_pages, n_kv_heads, head_dim, page_size] view of K."""
        return self.k_phys.permute(0, 1, 3, 2)

    @property
    def v_pages(self) -> torch.Tensor:
        return self.v_phys.permute(0, 1, 3, 2)

    def get_page_k(self, page_id: int) -> torch.Tensor:
        return self.k_pages[page_id]

    def get_page_v(self, page_id: int) -> torch.Tensor:
        return self.v_pages[page_id]

    @property
    def num_slots(self) -> int:
        return self.total_pages * self.config.page_size


class KVRequestCache:
    """Per-request block table + length + chunk keys (src/plastic_infer/kv/kv_store.py:98-182)."""

    def __init__(self, store: "KVStore", request_id: int = 0) -> None:
        self.store = store
        self.request_id = request_id
        self.cfg = store.config
        self.block_table = BlockTable(n_layers=self.cfg.n_layers, page_size=self.cfg.page_size)
        self._length = 0
        self.chunk_keys: list[ChunkKey] = []
        self._final_hash: Optional[bytes] = None
        # Leading complete chunks whose device pages evict_chunks released: their K/V
        # live only in the host store, and their block-table entries are -1.
        self.evicted_chunks = 0
        # token ids after the last complete chunk (extend_token_ids)
        self._token_tail: list[int] = []

    @property
    def length(self) -> int:
        return self._length

    def num_complete_chunks(self) -> int:
        return self._length // self.cfg.tokens_per_chunk

    def _ensure_page(self, pos: int) -> None:
        page_idx = pos // self.cfg.page_size
        for layer in range(self.cfg.n_layers):
            if self.block_table.num_logical_pages(layer) <= page_idx:
                self.block_table.append_page(layer, self.store.gpu.allocator.alloc())

    def reserve_tokens(self, n_tokens: int) -> None:
        """Allocate pages for the next n_tokens positions and advance the length
        without writing data (the caller writes every reserved slot afterwards).

        Replaces the reference's zero "dummy" appends before a forward pass
        (src/plastic_infer/exec/runner_paged.py:98-109, 222-226): those zeros are
        always overwritten by _write_kv_layer, so skipping them leaves the same pool.
        """
        if n_tokens <= 0:
            return
        S = self.cfg.page_size
        # Pages in the order the reference's per-token appends take them: page p of every
        # layer (layer 0 first), then page p + 1, ...
        for page_idx in range(self._length // S, (self._length + n_tokens - 1) // S + 1):
            self._ensure_page(page_idx * S)
        self._length += n_tokens

    def append_token(self, k_token: torch.Tensor, v_token: torch.Tensor) -> None:
        """Append one token's K/V for all layers; k_token, v_token: [n_layers, n_kv_heads, head_dim]."""
        cfg = self.cfg
        pos = self._length
        self._ensure_page(pos)
        gpu = self.store.gpu
        slots = [self.block_table.slot(layer, pos) for layer in range(cfg.n_layers)]
        slot_t = torch.tensor(slots, dtype=torch.int64, device=gpu.device)
        kernels.kv_index_copy(gpu.k_phys, gpu.v_phys, k_token.to(gpu.dtype), v_token.to(gpu.dtype),
                              slot_t)
        self._length += 1

    def set_token_ids(self, token_ids: list[int]) -> None:
        n_full = len(token_ids) // self.cfg.tokens_per_chunk
        self._token_tail = list(token_ids[n_full * self.cfg.tokens_per_chunk:])
        if n_full == 0:
            self.chunk_keys = []
            self._final_hash = None
            return
        keys, final_h = compute_prefix_hashes_and_final(
            token_ids[:n_full * self.cfg.tokens_per_chunk], chunk_size=self.cfg.tokens_per_chunk)
        self.chunk_keys = keys
        self._final_hash = final_h

    def extend_token_ids(self, token_ids: list[int]) -> int:
        """Append token ids (e.g. the ones a decode step generated) after those given so
        far; every chunk they complete gets its key, the same key set_token_ids over the
        whole sequence gives. Returns the number of chunk keys added (no reference
        counterpart: the reference recomputes every key with set_token_ids)."""
        tpc = self.cfg.tokens_per_chunk
        self._token_tail.extend(int(t) for t in token_ids)
        added = 0
        while len(self._token_tail) >= tpc:
            key = next_chunk_key(self._final_hash, self._token_tail[:tpc])
            self.chunk_keys.append(key)
            self._final_hash = key.cumulative_key
            del self._token_tail[:tpc]
            added += 1
        return added

    def get_block_table_for_layer(self, layer: int) -> list[int]:
        return list(self.block_table.pages[layer])


class _PinnedChunkPool:
    """Recycled pinned host buffers for chunks, physically [L, H, T, D] each."""

    def __init__(self, shape: tuple[int, ...], dtype: torch.dtype, pin: bool) -> None:
        self.shape = shape
        self.dtype = dtype
        self.pin = pin
        self._free: list[torch.Tensor] = []

    def take(self) -> torch.Tensor:
        if self._free:
            return self._free.pop()
        return torch.empty(self.shape, dtype=self.dtype, pin_memory=self.pin)

    def give(self, buf: torch.Tensor) -> None:
        self._free.append(buf)


class KVStore:
    """Device page pool + host chunk cache + prefix lookup (src/plastic_infer/kv/kv_store.py:185-406)."""

    def __init__(self, config: KVConfig) -> None:
        self.config = config
        self.gpu = KVPagedStorage(config, total_pages=config.max_pages,
                                  device=config.device, dtype=config.dtype)
        # full_key -> (k_chunk, v_chunk) logical views [L, H, D, T] of pinned buffers
        self._host_cache: dict[bytes, tuple[torch.Tensor, torch.Tensor]] = {}
        self._host_phys: dict[bytes, tuple[torch.Tensor, torch.Tensor]] = {}
        self._host_lru: OrderedDict[bytes, None] = OrderedDict()
        self._max_host_chunks = config.max_host_chunks
        self._prefix_index: dict[bytes, ChunkKey] = {}
        # host chunks that a live request has evicted from the device: not LRU-evictable
        self._host_pins: dict[bytes, int] = {}
        c = config
        on_cuda = self.gpu.device.type == "cuda"
        self._chunk_pool = _PinnedChunkPool(
            (c.n_layers, c.n_kv_heads, c.tokens_per_chunk, c.head_dim), c.dtype, pin=on_cuda)
        self._copy_stream: Optional[torch.cuda.Stream] = (
            torch.cuda.Stream(device=self.gpu.device) if on_cuda else None)
        # Sinks run on the side stream without blocking the caller: the event of the
        # latest one, and per host chunk the event after which its buffer holds the data.
        self._pending_sink: Optional[torch.cuda.Event] = None
        self._host_ready: dict[bytes, torch.cuda.Event] = {}

    # -- request lifecycle -------------------------------------------------------

    def new_request(self, request_id: int = 0) -> KVRequestCache:
        return KVRequestCache(self, request_id=request_id)

    def free_request(self, cache: KVRequestCache) -> None:
        self._order_page_reuse()
        self.gpu.allocator.free_many([p for p in cache.block_table.all_page_ids() if p >= 0])
        for c in range(min(cache.evicted_chunks, len(cache.chunk_keys))):
            self._unpin_host(cache.chunk_keys[c].full_key)
        cache.evicted_chunks = 0

    # -- sinking (device -> host) -------------------------------------------------

    def _chunk_page_list(self, cache: KVRequestCache, chunk_idx: int) -> list[int]:
        """Page ids of one chunk in (layer, page) order. A complete chunk always has
        all of them (reference, kv_store.py:261-262, skips missing ones)."""
        cfg = self.config
        start = chunk_idx * cfg.pages_per_chunk
        ids = []
        for layer in range(cfg.n_layers):
            for j in range(cfg.pages_per_chunk):
                ids.append(cache.block_table.get_page(layer, start + j))
        return ids

    def sink_completed_chunks(self, cache: KVRequestCache) -> int:
        """Copy every completed, not-yet-cached chunk to the host store.

        Same decisions as the reference (src/plastic_infer/kv/kv_store.py:230-276):
        cached chunks are only touched in the LRU, the host LRU is evicted to make
        room, and the return value counts newly sunk chunks. The copy is batched:
        one gather launch for all new chunks, one device->host copy per chunk on the
        store's side stream; like the reference's, this call returns once the host
        copies are complete (sink_completed_chunks_async does not wait).
        """
        n, ev = self.sink_completed_chunks_async(cache)
        if ev is not None:
            ev.synchronize()
        return n

    def sink_completed_chunks_async(self, cache: KVRequestCache
                                    ) -> tuple[int, Optional[torch.cuda.Event]]:
        """sink_completed_chunks without the wait (no reference counterpart).

        The gather and the device->host copies are queued on the store's side stream,
        after the work already queued on the current stream, and the call returns at
        once with (newly sunk chunks, event); the new host chunks hold their data once
        the event has completed. The store orders its own later work after it: attention
        over the chunks (host_stream_chunks) waits for the event on the GPU, and device
        pages freed by evict_chunks / free_request are reused only after the gather that
        reads them. Code that reads `_host_cache` tensors on the host must wait for the
        event first.
        """
        cfg = self.config
        todo: list[tuple[int, ChunkKey]] = []
        for chunk_idx, key in enumerate(cache.chunk_keys):
            full_key = key.full_key
            if full_key in self._host_cache:
                self._touch_host(full_key)
                continue
            if chunk_idx < cache.evicted_chunks:
                continue  # its device pages are gone: nothing left to copy
            while len(self._host_cache) >= self._max_host_chunks:
                if not self._evict_host_lru():
                    break  # every cached chunk is held by a live request
            todo.append((chunk_idx, key))
            # Reserve the LRU slot now so later chunks of this call evict correctly.
            self._host_cache[full_key] = (None, None)  # type: ignore[assignment]
            self._prefix_index[full_key] = key
            self._touch_host(full_key)
        # A chunk reserved above may already have been pushed out of the host LRU by a
        # later one of the same call (more new chunks than max_host_chunks); the
        # reference copies and then drops it, here it is simply not copied.
        live = [(i, key) for i, key in todo if key.full_key in self._host_cache]
        ev = None
        if live:
            page_ids: list[int] = []
            for chunk_idx, _ in live:
                page_ids += self._chunk_page_list(cache, chunk_idx)
            bufs, ev = self._move_out(page_ids, len(live))
            for (_, key), (kb, vb) in zip(live, bufs):
                self._host_phys[key.full_key] = (kb, vb)
                self._host_cache[key.full_key] = (kb.permute(0, 1, 3, 2), vb.permute(0, 1, 3, 2))
                self._host_ready[key.full_key] = ev
            self._pending_sink = ev
        return len(todo), ev

    def _order_page_reuse(self) -> None:
        """Before device pages are freed: later work on the current stream (which may
        write into the pages once they are handed out again) waits for the side-stream
        gathers of the sinks queued so far, which may still read them."""
        if self._pending_sink is not None and self.gpu.device.type == "cuda":
            torch.cuda.current_stream(self.gpu.device).wait_event(self._pending_sink)
            self._pending_sink = None

    def _move_out(self, page_ids: list[int], n_chunks: int
                  ) -> tuple[list[tuple[torch.Tensor, torch.Tensor]], torch.cuda.Event]:
        """Gather pages (ordered chunk, layer, page) into pinned chunk buffers, on the
        side stream; returns the buffers and the event that completes the copies."""
        cfg = self.config
        dev = self.gpu.device
        if dev.type != "cuda":
            raise RuntimeError("host-store page moves need a CUDA pool (no CPU path)")
        ids = torch.tensor(page_ids, dtype=torch.int32, device=dev)
        chunk_shape = self._chunk_pool.shape
        staging_k = torch.empty((n_chunks, *chunk_shape), dtype=cfg.dtype, device=dev)
        staging_v = torch.empty_like(staging_k)
        outs = [(self._chunk_pool.take(), self._chunk_pool.take()) for _ in range(n_chunks)]
        side = self._copy_stream
        main = torch.cuda.current_stream(dev)
        side.wait_stream(main)  # pool writes queued on the compute stream come first
        with torch.cuda.stream(side):
            kernels.page_gather(self.gpu.k_phys, ids, staging_k, pages_per_group=cfg.pages_per_chunk)
            kernels.page_gather(self.gpu.v_phys, ids, staging_v, pages_per_group=cfg.pages_per_chunk)
            for c, (kb, vb) in enumerate(outs):
                kb.copy_(staging_k[c], non_blocking=True)
                vb.copy_(staging_v[c], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(side)
        for t in (ids, staging_k, staging_v):
            t.record_stream(side)
        return outs, ev

    # -- prefix loading (host -> device) ------------------------------------------

    def load_prefix(self, cache: KVRequestCache, tokens: list[int]
                    ) -> tuple[int, list[ChunkKey]]:
        """Load the longest cached prefix of `tokens` into fresh pages.

        Same allocation order, eviction trigger and cache state updates as the
        reference (src/plastic_infer/kv/kv_store.py:282-334); the data move is one
        host->device copy per chunk plus one scatter launch per pool, on the side
        stream, with the compute stream ordered after it.
        """
        cfg = self.config
        matches, _ = longest_prefix_hits(self._prefix_index, tokens, chunk_size=cfg.tokens_per_chunk)
        if not matches:
            return 0, []
        matched_tokens = len(matches) * cfg.tokens_per_chunk
        need = len(matches) * cfg.n_layers * cfg.pages_per_chunk
        if self.gpu.allocator.free_pages < need:
            self.evict_chunks(need - self.gpu.allocator.free_pages)
        page_ids: list[int] = []
        for _ in matches:
            for layer in range(cfg.n_layers):
                for _j in range(cfg.pages_per_chunk):
                    pid = self.gpu.allocator.alloc()
                    cache.block_table.append_page(layer, pid)
                    page_ids.append(pid)
        self._move_in(page_ids, [self._host_phys[m.full_key] for m in matches])
        cache._length = matched_tokens
        cache.chunk_keys = list(matches)
        cache._final_hash = matches[-1].cumulative_key
        for key in matches:
            self._touch_host(key.full_key)
        return matched_tokens, matches

    def _move_in(self, page_ids: list[int], chunks: list[tuple[torch.Tensor, torch.Tensor]]) -> None:
        cfg = self.config
        dev = self.gpu.device
        if dev.type != "cuda":
            raise RuntimeError("host-store page moves need a CUDA pool (no CPU path)")
        n = len(chunks)
        staging_k = torch.empty((n, *self._chunk_pool.shape), dtype=cfg.dtype, device=dev)
        staging_v = torch.empty_like(staging_k)
        ids = torch.tensor(page_ids, dtype=torch.int32, device=dev)
        side = self._copy_stream
        main = torch.cuda.current_stream(dev)
        side.wait_stream(main)
        with torch.cuda.stream(side):
            for c, (kb, vb) in enumerate(chunks):
                staging_k[c].copy_(kb, non_blocking=True)
                staging_v[c].copy_(vb, non_blocking=True)
            kernels.page_scatter(staging_k, ids, self.gpu.k_phys, pages_per_group=cfg.pages_per_chunk)
            kernels.page_scatter(staging_v, ids, self.gpu.v_phys, pages_per_group=cfg.pages_per_chunk)
        for t in (ids, staging_k, staging_v):
            t.record_stream(side)
        main.wait_stream(side)

    # -- eviction (device) ----------------------------------------------------------

    def evict_chunks(self, need_pages: int,
                     protected_request: Optional[KVRequestCache] = None) -> int:
        """Free the device pages of the oldest complete chunks of `protected_request`.

        The reference's v1 policy (src/plastic_infer/kv/kv_store.py:340-386): oldest
        chunk first, the newest complete chunk is always kept, stop once `need_pages`
        pages are freed; returns the pages freed (0 without a protected request).

        Fixed here: the reference leaves freed pages in the request's block table
        (kv_store.py:380-383), so a second call frees them again (the allocator's
        double-free assertion) and attention would read pages that now belong to
        another request. Here an evicted chunk's block-table entries become -1, the
        request counts its leading evicted chunks (`evicted_chunks`) and a later call
        continues after them, and the chunk's host copy (if it was sunk) is held in
        the host LRU while the request lives. Attention over such a request reads the
        host copies in place: host_stream_attention_v1(q, *store.host_stream_chunks(
        cache, layer), ...). Evicting a chunk that was never sunk loses its K/V, as in
        the reference; host_stream_chunks then raises.
        """
        if protected_request is None:
            return 0
        cfg = self.config
        cache = protected_request
        freed = 0
        self._order_page_reuse()
        n_full = cache.num_complete_chunks()
        while cache.evicted_chunks < n_full - 1 and freed < need_pages:
            c = cache.evicted_chunks
            start = c * cfg.pages_per_chunk
            pages: list[int] = []
            for layer in range(cfg.n_layers):
                row = cache.block_table.pages[layer]
                for j in range(cfg.pages_per_chunk):
                    lp = start + j
                    if lp < len(row) and row[lp] >= 0:
                        pages.append(row[lp])
                        row[lp] = -1
            self.gpu.allocator.free_many(pages)
            freed += len(pages)
            if c < len(cache.chunk_keys):
                self._pin_host(cache.chunk_keys[c].full_key)
            cache.evicted_chunks += 1
        return freed

    def host_stream_chunks(self, cache: KVRequestCache, layer: int,
                           device_table: Optional[torch.Tensor] = None
                           ) -> tuple[list[tuple[torch.Tensor, torch.Tensor]], torch.Tensor, torch.Tensor]:
        """The KV of one layer of `cache` as host_stream_attention_v1 takes it.

        Returns (host_chunks, resident_k, resident_v). host_chunks holds the host copies
        of the request's evicted chunks, oldest first, as [H_kv, D, C] views of the
        pinned chunk buffers: the kernel reads them in place, nothing is copied back.
        resident_k / resident_v [1, R, H_kv, D] are the tokens still in the device pool,
        gathered in one launch each. `device_table`, when given, is this layer's block
        table row of the request already on the device (int32, at least as long as the
        row; entries of evicted chunks are not read); otherwise the row is copied from
        the host list.
        """
        cfg = self.config
        chunks: list[tuple[torch.Tensor, torch.Tensor]] = []
        waited: list[torch.cuda.Event] = []
        for c in range(cache.evicted_chunks):
            key = cache.chunk_keys[c].full_key if c < len(cache.chunk_keys) else None
            kv = self._host_cache.get(key) if key is not None else None
            if kv is None or kv[0] is None:
                raise RuntimeError(f"chunk {c} left the device pool without a host copy")
            chunks.append((kv[0][layer], kv[1][layer]))
            ready = self._host_ready.get(key)
            if ready is not None and ready not in waited:
                # the kernel reads the host buffer in place: after its sink's copies
                torch.cuda.current_stream(self.gpu.device).wait_event(ready)
                waited.append(ready)
        start = cache.evicted_chunks * cfg.pages_per_chunk
        n_tail = cache.length - cache.evicted_chunks * cfg.tokens_per_chunk
        dev = self.gpu.device
        if device_table is not None:
            bt = device_table[start:]
        else:
            table = cache.block_table.pages[layer][start:]
            bt = torch.tensor(table if table else [0], dtype=torch.int32, device=dev)
        rk = kernels.paged_kv_gather(self.gpu.k_phys, bt, n_tail).unsqueeze(0)
        rv = kernels.paged_kv_gather(self.gpu.v_phys, bt, n_tail).unsqueeze(0)
        return chunks, rk, rv

    def _pin_host(self, full_key: bytes) -> None:
        if full_key in self._host_cache:
            self._host_pins[full_key] = self._host_pins.get(full_key, 0) + 1

    def _unpin_host(self, full_key: bytes) -> None:
        n = self._host_pins.get(full_key, 0)
        if n <= 1:
            self._host_pins.pop(full_key, None)
        else:
            self._host_pins[full_key] = n - 1

    # -- host LRU -------------------------------------------------------------------

    def _touch_host(self, full_key: bytes) -> None:
        if full_key in self._host_lru:
            del self._host_lru[full_key]
        self._host_lru[full_key] = None

    def _evict_host_lru(self) -> bool:
        """Drop the least recently used host chunk that no live request holds; False
        when there is none."""
        oldest = next((k for k in self._host_lru if k not in self._host_pins), None)
        if oldest is None:
            return False
        del self._host_lru[oldest]
        del self._host_cache[oldest]
        self._host_ready.pop(oldest, None)
        self._prefix_index.pop(oldest, None)
        phys = self._host_phys.pop(oldest, None)
        if phys is not None:
            self._chunk_pool.give(phys[0])
            self._chunk_pool.give(phys[1])
        return True

    def has_host_chunk(self, full_key: bytes) -> bool:
        """Whether the host store holds (or is being sent) the chunk with this key."""
        return full_key in self._host_cache

    def host_chunk(self, full_key: bytes
                   ) -> tuple[torch.Tensor, torch.Tensor, Optional[torch.cuda.Event]]:
        """The host copy of a chunk: (k, v) logical [L, H_kv, D, T] views of its pinned
        buffers and the event after which they hold the data (None once known complete)."""
        kv = self._host_cache.get(full_key)
        if kv is None or kv[0] is None:
            raise KeyError("no host copy of this chunk")
        return kv[0], kv[1], self._host_ready.get(full_key)

    @property
    def host_cache_size(self) -> int:
        return len(self._host_cache)
