"""CPU oracle of plastic-infer's paged-KV decode hot path (numpy restatement).

TEST INFRASTRUCTURE ONLY. This module is the parity checker: only tests/,
__graft_entry__.smoke() and bench.py's CPU baseline / reference arm may import it.
The product path (plastic_infer_b200) never calls it and has no CPU fallback.

Every function restates the reference algorithm in plain numpy and cites the
reference line it follows (paths relative to the plastic-infer project). The
restatement is pinned against golden vectors produced by running the reference
itself (tests/golden/make_golden.py; checked by tests/test_oracle_golden.py).

Layouts are the reference's *logical* ones:
  page pool  [num_pages, kv_heads, head_dim, page_size]   (src/plastic_infer/kv/kv_store.py:86-88)
  host chunk [n_layers, kv_heads, head_dim, tokens_per_chunk] (src/plastic_infer/kv/kv_store.py:252-256)
bf16 data is carried as uint16 bit patterns (numpy has no bfloat16), so byte copies
stay bit-exact and arithmetic widens to float32 first.
"""

from __future__ import annotations

import hashlib

import numpy as np

# ---------------------------------------------------------------------------
# bf16 bit helpers
# ---------------------------------------------------------------------------


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 (round-to-nearest-even), returned as uint16 bits.

    Same rounding as torch's float32 -> bfloat16 conversion for finite values.
    """
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out = np.where(nan, np.uint16(0x7FC0), out)
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------
# a1: slot-mapping KV write
# ---------------------------------------------------------------------------


def slot_of(block_table_layer: list[int], token: int, page_size: int) -> int:
    """Flat slot of a token: page id * page_size + offset.

    BlockTable.get_page / get_page_for_token (src/plastic_infer/kv/paged.py:54-59)
    and the page_idx/page_off arithmetic of _write_kv_layer
    (src/plastic_infer/exec/runner_paged.py:124-127).
    """
    return block_table_layer[token // page_size] * page_size + token % page_size


def write_kv_slots(k_pages: np.ndarray, v_pages: np.ndarray, k_new: np.ndarray,
                   v_new: np.ndarray, slots: np.ndarray, page_size: int) -> None:
    """In place: pool[slot // S, :, :, slot % S] = new[i] for each slot >= 0.

    The per-token assignment of _write_kv_layer (src/plastic_infer/exec/runner_paged.py:128-129)
    and KVRequestCache.append_token (src/plastic_infer/kv/kv_store.py:142-143), applied in
    token order so a repeated slot keeps the last write. Negative slots are padding.
    """
    for i, s in enumerate(np.asarray(slots, dtype=np.int64)):
        if s < 0:
            continue
        page, off = divmod(int(s), page_size)
        k_pages[page, :, :, off] = k_new[i]
        v_pages[page, :, :, off] = v_new[i]


# ---------------------------------------------------------------------------
# a2: paged decode attention
# ---------------------------------------------------------------------------


def gather_paged_kv(k_pages: np.ndarray, v_pages: np.ndarray, block_table: list[int],
                    page_size: int, num_tokens: int | None = None):
    """Contiguous [T, kv_heads, head_dim] K and V of one request.

    gather_paged_kv (src/plastic_infer/exec/attention.py:103-148): index_select the
    pages, permute [n, H, D, S] -> [n, S, H, D], flatten, trim to num_tokens.
    """
    H, D = k_pages.shape[1], k_pages.shape[2]
    if len(block_table) == 0:
        e = np.zeros((0, H, D), dtype=k_pages.dtype)
        return e, e.copy()
    ids = np.asarray(block_table, dtype=np.int64)
    k = k_pages[ids].transpose(0, 3, 1, 2).reshape(len(ids) * page_size, H, D)
    v = v_pages[ids].transpose(0, 3, 1, 2).reshape(len(ids) * page_size, H, D)
    if num_tokens is not None:
        k, v = k[:num_tokens], v[:num_tokens]
    return k, v


def paged_attention_decode(q: np.ndarray, k_pages: np.ndarray, v_pages: np.ndarray,
                           block_tables: list[list[int]], ctx_lens, page_size: int,
                           scale: float | None = None) -> np.ndarray:
    """Batched single-token paged attention, fp32 arithmetic.

    For each request b: gather its first ctx_lens[b] tokens (attention.py:133-146),
    expand KV heads with query head h reading KV head h // G (attention.py:180-187),
    then softmax(q . K^T * scale) V with scale = 1/sqrt(D) (the SDPA default used at
    attention.py:189; causal masking is a no-op for one query token at the end of the
    context, as in decode, runner_paged.py:254-255). A request with no context
    yields zeros (SDPA over zero keys).

    q: [B, Hq, D]; pools logical fp32 (bf16 inputs widened by the caller).
    """
    q = np.asarray(q, dtype=np.float32)
    B, Hq, D = q.shape
    Hkv = k_pages.shape[1]
    G = Hq // Hkv
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    out = np.zeros((B, Hq, D), dtype=np.float32)
    for b in range(B):
        n = int(ctx_lens[b])
        if n <= 0:
            continue
        npg = -(-n // page_size)
        ids = np.asarray(block_tables[b][:npg], dtype=np.int64)
        # Gathered pages [npg, Hkv, D, S] -> per-head K^T / V^T [Hkv, D, T] (the same
        # token order as gather_paged_kv's permute + reshape), trimmed to n tokens.
        kt = k_pages[ids].astype(np.float32, copy=False).transpose(1, 2, 0, 3)
        vt = v_pages[ids].astype(np.float32, copy=False).transpose(1, 2, 0, 3)
        kt = kt.reshape(Hkv, D, npg * page_size)[:, :, :n]
        vt = vt.reshape(Hkv, D, npg * page_size)[:, :, :n]
        qg = q[b].reshape(Hkv, G, D)                          # query head h*G+g -> KV head h
        s = np.matmul(qg, kt) * np.float32(scale)             # [Hkv, G, n]
        s -= s.max(axis=2, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=2, keepdims=True)
        out[b] = np.matmul(p, vt.transpose(0, 2, 1)).reshape(Hq, D)
    return out


def paged_attention_prefill(q: np.ndarray, k_pages: np.ndarray, v_pages: np.ndarray,
                            block_table: list[int], kv_len: int, q_start: int, causal: bool,
                            page_size: int, scale: float | None = None) -> np.ndarray:
    """Prefill attention of one request: q [q_len, Hq, D] over its first kv_len tokens.

    src/plastic_infer/exec/runner_paged.py:36-95 (_attn_paged): query i sits at position
    q_start + i; causal -> it sees keys j < min(kv_len, q_start + i + 1). With q_start == 0
    that is SDPA's is_causal on the gathered context (attention.py:151-190, top-left
    aligned), with q_start > 0 the dense mask built at runner_paged.py:70-76; non-causal
    sees all kv_len keys. GQA head h reads KV head h // G. float64 softmax.
    """
    q = np.asarray(q, dtype=np.float64)
    L, Hq, D = q.shape
    if kv_len == 0:
        return np.zeros((L, Hq, D), dtype=np.float32)
    k, v = gather_paged_kv(k_pages, v_pages, block_table, page_size, kv_len)  # [kv, H, D]
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    Hkv = k.shape[1]
    G = Hq // Hkv
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    kh = np.repeat(k, G, axis=1).transpose(1, 0, 2)      # [Hq, kv, D]
    vh = np.repeat(v, G, axis=1).transpose(1, 0, 2)
    s = np.einsum("lhd,hjd->hlj", q, kh) * scale          # [Hq, L, kv]
    j = np.arange(kv_len)[None, :]
    lim = np.minimum(kv_len, q_start + np.arange(L) + 1)[:, None] if causal else np.full((L, 1), kv_len)
    s = np.where(j < lim, s, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("hlj,hjd->lhd", p, vh).astype(np.float32)


def host_stream_attention(q: np.ndarray, host_chunks: list[tuple[np.ndarray, np.ndarray]],
                          resident_k: np.ndarray, resident_v: np.ndarray, q_start: int = 0,
                          causal: bool = True, scale: float | None = None) -> np.ndarray:
    """Attention over host chunks plus a resident tail (one request).

    src/plastic_infer/exec/attention.py:193-250 (host_stream_attention_v1): the chunks
    ([H_kv, D, C] each, oldest first) and the tail ([1, R, H_kv, D]) are concatenated
    into [1, kv_len, H_kv, D]; query row i of q [1, q_len, Hq, D] sits at position
    q_start + i. causal -> it sees keys j <= q_start + i (the dense mask of :236-243, and
    SDPA's is_causal when q_start == 0 and q_len == kv_len, which is the same set);
    non-causal sees every key. GQA head h reads KV head h // G. float64 softmax; rows
    with no visible key (kv_len == 0) are zero.
    """
    q = np.asarray(q, dtype=np.float64)[0]                       # [L, Hq, D]
    parts_k = [np.asarray(kc, dtype=np.float64).transpose(2, 0, 1) for kc, _ in host_chunks]
    parts_v = [np.asarray(vc, dtype=np.float64).transpose(2, 0, 1) for _, vc in host_chunks]
    k = np.concatenate(parts_k + [np.asarray(resident_k, dtype=np.float64)[0]], axis=0)
    v = np.concatenate(parts_v + [np.asarray(resident_v, dtype=np.float64)[0]], axis=0)
    L, Hq, D = q.shape
    kv_len, Hkv = k.shape[0], k.shape[1]
    if kv_len == 0:
        return np.zeros((1, L, Hq, D), dtype=np.float32)
    G = Hq // Hkv
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    kh = np.repeat(k, G, axis=1).transpose(1, 0, 2)              # [Hq, kv, D]
    vh = np.repeat(v, G, axis=1).transpose(1, 0, 2)
    s = np.einsum("lhd,hjd->hlj", q, kh) * scale                 # [Hq, L, kv]
    if causal:
        j = np.arange(kv_len)[None, :]
        s = np.where(j <= q_start + np.arange(L)[:, None], s, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    p_ = np.exp(s)
    p_ /= p_.sum(axis=-1, keepdims=True)
    return np.einsum("hlj,hjd->lhd", p_, vh)[None].astype(np.float32)


# ---------------------------------------------------------------------------
# Decode prologue: QK-norm + RoPE of the step's q / k rows (then the slot write above)
# ---------------------------------------------------------------------------


def rms_norm_rows(x: np.ndarray, weight: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """x / sqrt(mean(x^2) + eps) * weight over the last axis, in float32.

    src/plastic_infer/exec/attention.py:77-80 (rms_norm), applied per head as qk_norm does
    (attention.py:83-95: the norm acts over head_dim, before RoPE).
    """
    x = np.asarray(x, dtype=np.float32)
    rms = np.sqrt(np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32) + np.float32(eps))
    return (x / rms * np.asarray(weight, dtype=np.float32)).astype(np.float32)


def rope_rows(x: np.ndarray, positions: np.ndarray, inv_freq: np.ndarray) -> np.ndarray:
    """Rotary embedding of x [B, H, D] at per-request positions [B], in float32.

    src/plastic_infer/exec/attention.py:23-49 (rope_positions: x * cos + rotate_half(x) *
    sin, rotate_half = cat(-x2, x1)) over the table of attention.py:52-74
    (cos/sin of cat(freqs, freqs), freqs = outer(t, inv_freq)): the angle of (pos, j) is
    the float32 product pos * inv_freq[j mod D/2].
    """
    x = np.asarray(x, dtype=np.float32)
    half = x.shape[-1] // 2
    ang = (np.asarray(positions, dtype=np.float32)[:, None] * np.asarray(inv_freq, np.float32)[None, :])
    ang = np.concatenate([ang, ang], axis=-1).astype(np.float32)
    cos = np.cos(ang.astype(np.float64)).astype(np.float32)[:, None, :]
    sin = np.sin(ang.astype(np.float64)).astype(np.float32)[:, None, :]
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return (x * cos + rot * sin).astype(np.float32)


def decode_prologue(q: np.ndarray, k: np.ndarray, v: np.ndarray, positions: np.ndarray,
                    inv_freq: np.ndarray, q_norm_w: np.ndarray | None = None,
                    k_norm_w: np.ndarray | None = None, eps: float = 1e-5):
    """(q_rot, k_rot, v) of one decode step: optional QK-norm, then RoPE on q and k.

    The order of the reference's MoE runner (src/plastic_infer/exec/runner_moe_paged.py:135-142:
    qk_norm, then rope_positions); the dense runner has no QK-norm
    (src/plastic_infer/exec/runner_paged.py:247-248). The K/V rows then go to their slots
    as write_kv_slots does.
    """
    if q_norm_w is not None:
        q = rms_norm_rows(q, q_norm_w, eps)
        k = rms_norm_rows(k, k_norm_w, eps)
    return rope_rows(q, positions, inv_freq), rope_rows(k, positions, inv_freq), v


# ---------------------------------------------------------------------------
# MoE expert-slot copy (row gather by index, every bank)
# ---------------------------------------------------------------------------


def expert_slot_copy(dst_banks: list, src_banks: list, dst_idx: np.ndarray, src_idx: np.ndarray,
                     n: int | None = None) -> None:
    """dst_b[dst_idx[i]] = src_b[src_idx[i]] for every bank and i < n, in place.

    The per-bank semantics of the reference's fused multi-bank copy
    (src/plastic_infer/kernel/csrc/jit/fast_index_copy.cuh:448-472: row u // units of
    src_indices, 16-byte units of the row) and of copy_missing's pageable path
    (src/plastic_infer/moe/offload_cache.py:992-996: index_select + index_copy_). Banks are
    2-D arrays [rows, feature]; destination rows must be distinct.
    """
    n = len(dst_idx) if n is None else min(int(n), len(dst_idx))
    for dst, src in zip(dst_banks, src_banks):
        dst[np.asarray(dst_idx[:n], dtype=np.int64)] = src[np.asarray(src_idx[:n], dtype=np.int64)]


# ---------------------------------------------------------------------------
# a3: page moves between the pool and host chunks
# ---------------------------------------------------------------------------


def sink_chunk(k_pages: np.ndarray, v_pages: np.ndarray, block_table: list[list[int]],
               chunk_idx: int, page_size: int, pages_per_chunk: int):
    """Host copy of one completed chunk, [L, H, D, page_size * pages_per_chunk].

    KVStore.sink_completed_chunks (src/plastic_infer/kv/kv_store.py:250-269): for each
    layer and each page of the chunk, k_chunk[layer, :, :, t0:t1] = k_pages[phys].
    Pages missing from a layer's table stay zero (kv_store.py:261-262).
    """
    L = len(block_table)
    H, D = k_pages.shape[1], k_pages.shape[2]
    T = page_size * pages_per_chunk
    kc = np.zeros((L, H, D, T), dtype=k_pages.dtype)
    vc = np.zeros((L, H, D, T), dtype=v_pages.dtype)
    start = chunk_idx * pages_per_chunk
    for layer in range(L):
        for j in range(pages_per_chunk):
            lp = start + j
            if lp >= len(block_table[layer]):
                continue
            phys = block_table[layer][lp]
            kc[layer, :, :, j * page_size:(j + 1) * page_size] = k_pages[phys]
            vc[layer, :, :, j * page_size:(j + 1) * page_size] = v_pages[phys]
    return kc, vc


def load_chunk(k_pages: np.ndarray, v_pages: np.ndarray, k_chunk: np.ndarray,
               v_chunk: np.ndarray, phys_pages: list[list[int]], page_size: int) -> None:
    """In place: pool[phys_pages[l][j]] = chunk[l, :, :, j*S:(j+1)*S].

    KVStore.load_prefix's copy loop (src/plastic_infer/kv/kv_store.py:311-321).
    """
    for layer, pages in enumerate(phys_pages):
        for j, phys in enumerate(pages):
            k_pages[phys] = k_chunk[layer, :, :, j * page_size:(j + 1) * page_size]
            v_pages[phys] = v_chunk[layer, :, :, j * page_size:(j + 1) * page_size]


# ---------------------------------------------------------------------------
# chunk keys (host-store addressing)
# ---------------------------------------------------------------------------

INITIAL_SALT = b"plastic-infer-kv-v1"


def chunk_keys(tokens: list[int], chunk_size: int) -> list[tuple[bytes, bytes]]:
    """(prefix_key, cumulative_key) per chunk.

    _compute_hashes (src/plastic_infer/kv/chunk.py:80-111): h0 = sha256(salt);
    c_i = sha256 of the chunk's tokens as 4-byte little-endian unsigned ints;
    h_{i+1} = sha256(h_i || c_i).
    """
    if len(tokens) % chunk_size:
        raise ValueError("token count not aligned to chunk_size")
    running = hashlib.sha256(INITIAL_SALT).digest()
    keys = []
    for c in range(len(tokens) // chunk_size):
        ch = hashlib.sha256(
            b"".join(int(t).to_bytes(4, "little", signed=False)
                     for t in tokens[c * chunk_size:(c + 1) * chunk_size])).digest()
        cum = hashlib.sha256(running + ch).digest()
        keys.append((running, cum))
        running = cum
    return keys
