"""Page allocator and per-request block table (host-side addressing).

Same interface and behaviour as the reference's kv/paged.py
(src/plastic_infer/kv/paged.py:25-160): a LIFO free list of global page ids shared by
all layers, and a per-request table mapping (layer, logical page) -> page id. The
LIFO order is kept exactly, so a sequence of requests gets the same page ids as in
the reference (pinned by tests/golden/allocator.json).

Additions for the batched device path: `BlockTable.page_ids_tensor` returns a
layer's table as an int32 tensor, and `slots_for` resolves token positions to
flat slots (page_id * page_size + offset) for the index-copy kernel.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

DEFAULT_PAGE_SIZE: int = 16   # tokens per page (src/plastic_infer/kv/paged.py:25)
DEFAULT_CHUNK_PAGES: int = 16  # pages per host chunk (src/plastic_infer/kv/paged.py:26)


@dataclass
class BlockTable:
    """pages[layer][i] = page id holding logical tokens [i*page_size, (i+1)*page_size)."""

    n_layers: int
    page_size: int
    pages: list[list[int]] = field(default_factory=list)

    def __post_init__(self) -> None:
        if not self.pages:
            self.pages = [[] for _ in range(self.n_layers)]

    def num_logical_pages(self, layer: int) -> int:
        return len(self.pages[layer])

    def num_tokens(self, layer: int) -> int:
        return len(self.pages[layer]) * self.page_size

    def get_page(self, layer: int, logical_page_idx: int) -> int:
        return self.pages[layer][logical_page_idx]

    def get_page_for_token(self, layer: int, token_idx: int) -> int:
        return self.pages[layer][token_idx // self.page_size]

    def append_page(self, layer: int, phys_page_id: int) -> None:
        self.pages[layer].append(phys_page_id)

    def all_page_ids(self) -> set[int]:
        out: set[int] = set()
        for row in self.pages:
            out.update(row)
        return out

    def chunk_page_ids(self, chunk_idx: int, pages_per_chunk: int) -> list[int]:
        lo = chunk_idx * pages_per_chunk
        hi = lo + pages_per_chunk
        return [pid for row in self.pages for pid in row[lo:min(hi, len(row))]]

    def is_chunk_complete(self, chunk_idx: int, pages_per_chunk: int) -> bool:
        need = (chunk_idx + 1) * pages_per_chunk
        return all(len(row) >= need for row in self.pages)

    # -- batched-path helpers -------------------------------------------------

    def slot(self, layer: int, token_idx: int) -> int:
        """Flat pool slot of one token: page_id * page_size + offset."""
        return self.pages[layer][token_idx // self.page_size] * self.page_size + token_idx % self.page_size

    def slots_for(self, layer: int, start: int, count: int) -> list[int]:
        S = self.page_size
        row = self.pages[layer]
        return [row[t // S] * S + t % S for t in range(start, start + count)]

    def page_ids_tensor(self, layer: int, device: torch.device | str | None = None) -> torch.Tensor:
        return torch.tensor(self.pages[layer], dtype=torch.int32, device=device)


class PageAllocator:
    """LIFO free list of page ids 0..total_pages-1 (src/plastic_infer/kv/paged.py:96-160)."""

    def __init__(self, total_pages: int) -> None:
        assert total_pages > 0
        self._total = total_pages
        self._free: list[int] = list(range(total_pages - 1, -1, -1))  # pop() yields 0 first
        self._used: set[int] = set()

    @property
    def total_pages(self) -> int:
        return self._total

    @property
    def free_pages(self) -> int:
        return len(self._free)

    @property
    def used_pages(self) -> int:
        return self._total - len(self._free)

    def alloc(self) -> int:
        if not self._free:
            raise IndexError("out of pages")
        pid = self._free.pop()
        self._used.add(pid)
        return pid

    def alloc_many(self, count: int) -> list[int]:
        if count > len(self._free):
            raise IndexError(f"need {count} pages, only {len(self._free)} free")
        ids = [self._free.pop() for _ in range(count)]
        self._used.update(ids)
        return ids

    def free(self, page_id: int) -> None:
        assert page_id in self._used, f"page {page_id} not in use"
        self._used.discard(page_id)
        self._free.append(page_id)

    def free_many(self, page_ids: list[int]) -> None:
        for pid in page_ids:
            assert pid in self._used, f"page {pid} not in use"
            self._used.discard(pid)
        self._free.extend(page_ids)

    def is_used(self, page_id: int) -> bool:
        return page_id in self._used
