"""Paged KV storage, allocation and host chunk store (drop-in for plastic_infer.kv)."""

from .chunk import ChunkKey, compute_prefix_hashes, compute_prefix_hashes_and_final, longest_prefix_hits
from .kv_store import KVConfig, KVPagedStorage, KVRequestCache, KVStore
from .paged import DEFAULT_CHUNK_PAGES, DEFAULT_PAGE_SIZE, BlockTable, PageAllocator

__all__ = [
    "BlockTable", "ChunkKey", "DEFAULT_CHUNK_PAGES", "DEFAULT_PAGE_SIZE", "KVConfig",
    "KVPagedStorage", "KVRequestCache", "KVStore", "PageAllocator", "compute_prefix_hashes",
    "compute_prefix_hashes_and_final", "longest_prefix_hits",
]
