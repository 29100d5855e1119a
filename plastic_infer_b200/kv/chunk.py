"""Content-addressed chunk keys for the host KV store.

The key format must be byte-identical to the reference's so host chunks are
interchangeable: chained SHA-256 over 4-byte little-endian token ids with the salt
b"plastic-infer-kv-v1" (src/plastic_infer/kv/chunk.py:22, 80-111). Longest-prefix
matching follows src/plastic_infer/kv/chunk.py:114-149. Pinned by
tests/golden/chunk_keys.json.
"""

from __future__ import annotations

import hashlib
import struct
from dataclasses import dataclass

DEFAULT_CHUNK_SIZE: int = 256
_INITIAL_SALT = b"plastic-infer-kv-v1"


@dataclass(frozen=True)
class ChunkKey:
    prefix_key: bytes       # digest of everything before this chunk
    cumulative_key: bytes   # digest including this chunk

    def __repr__(self) -> str:
        return f"ChunkKey({self.cumulative_key.hex()[:16]})"

    @property
    def full_key(self) -> bytes:
        return self.cumulative_key


def _chain(tokens: list[int], chunk_size: int, salt: bytes) -> tuple[list[ChunkKey], bytes]:
    if len(tokens) % chunk_size != 0:
        raise ValueError(f"token count {len(tokens)} not aligned to chunk_size {chunk_size}")
    running = hashlib.sha256(salt).digest()
    keys: list[ChunkKey] = []
    for start in range(0, len(tokens), chunk_size):
        body = struct.pack(f"<{chunk_size}I", *tokens[start:start + chunk_size])
        cum = hashlib.sha256(running + hashlib.sha256(body).digest()).digest()
        keys.append(ChunkKey(prefix_key=running, cumulative_key=cum))
        running = cum
    return keys, running


def next_chunk_key(running: bytes | None, chunk_tokens: list[int],
                   initial_salt: bytes = _INITIAL_SALT) -> ChunkKey:
    """Key of the chunk that follows `running` (the previous chunk's cumulative key, or
    None for the first chunk): the step of the chain above, so keys built one chunk at a
    time equal compute_prefix_hashes over the whole sequence."""
    if running is None:
        running = hashlib.sha256(initial_salt).digest()
    body = struct.pack(f"<{len(chunk_tokens)}I", *chunk_tokens)
    return ChunkKey(prefix_key=running,
                    cumulative_key=hashlib.sha256(running + hashlib.sha256(body).digest()).digest())


def compute_prefix_hashes(tokens: list[int], chunk_size: int = DEFAULT_CHUNK_SIZE,
                          initial_salt: bytes = _INITIAL_SALT) -> list[ChunkKey]:
    return _chain(tokens, chunk_size, initial_salt)[0]


def compute_prefix_hashes_and_final(tokens: list[int], chunk_size: int = DEFAULT_CHUNK_SIZE,
                                    initial_salt: bytes = _INITIAL_SALT
                                    ) -> tuple[list[ChunkKey], bytes]:
    return _chain(tokens, chunk_size, initial_salt)


def longest_prefix_hits(cache_index: dict[bytes, ChunkKey], tokens: list[int],
                        chunk_size: int = DEFAULT_CHUNK_SIZE) -> tuple[list[ChunkKey], int]:
    """Longest run of whole leading chunks of `tokens` present in cache_index."""
    n_full = len(tokens) // chunk_size
    keys, _ = _chain(tokens[:n_full * chunk_size], chunk_size, _INITIAL_SALT)
    matched: list[ChunkKey] = []
    for key in keys:
        if key.full_key not in cache_index:
            break
        matched.append(key)
    return matched, len(matched) * chunk_size
