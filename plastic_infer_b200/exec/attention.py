"""Attention ops with the reference's signatures, backed by the sm_100a kernels.

Drop-in for src/plastic_infer/exec/attention.py:

* `gather_paged_kv`   -> pi_paged_kv_gather (one launch per pool) instead of
                         index_select + permute + reshape (attention.py:103-148).
* `paged_attention_v1`-> for a single query token (decode), the batched paged decode
                         kernel with B = 1 (no gather, no repeat_interleave, one pass
                         over the pages); for prefill (Sq > 1) the reference algorithm
                         (gather + SDPA) over the kernel gather. Paged prefill is not
                         part of the decode hot path.
* `host_stream_attention_v1` -> pi_host_stream_attn: one pass over the host chunks
                         (pinned ones read in place) and the resident tail, instead of
                         concatenating them and running SDPA (attention.py:193-250).
* RoPE / RMSNorm / QK-norm keep the reference math (attention.py:23-95); they are
  used by the runners, not by the KV path.

Pools may be passed as the logical [P, H, D, S] views that KVPagedStorage exposes
(zero-copy) or as any logical tensor (converted to the physical layout with a copy).
All tensors must be on a CUDA device: there is no CPU path.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import kernels


def rope_positions(cos: torch.Tensor, sin: torch.Tensor, positions: torch.Tensor,
                   x: torch.Tensor) -> torch.Tensor:
    """Rotary embedding with the rotate-half pairing (attention.py:23-49).

    cos/sin: [seq_len, head_dim]; positions: [S]; x: [B, S, H, head_dim].
    """
    c = cos.index_select(0, positions)[None, :, None, :]
    s = sin.index_select(0, positions)[None, :, None, :]
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * c + rot * s


def build_rope_cache(seq_len: int, head_dim: int, base: float = 10000.0,
                     device: torch.device | None = None,
                     dtype: torch.dtype = torch.float32) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin tables [seq_len, head_dim], frequencies repeated over both halves,
    computed in `dtype` like the reference (attention.py:52-74)."""
    exponents = torch.arange(0, head_dim, 2, dtype=dtype, device=device) / head_dim
    inv_freq = 1.0 / (base ** exponents)
    angles = torch.arange(seq_len, dtype=dtype, device=device)[:, None] * inv_freq[None, :]
    angles = torch.cat((angles, angles), dim=-1)
    return angles.cos(), angles.sin()


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """x / sqrt(mean(x^2) + eps) * weight (attention.py:77-80)."""
    return x / torch.sqrt((x * x).mean(dim=-1, keepdim=True) + eps) * weight


def qk_norm(q: torch.Tensor, k: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
            head_dim: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-head RMSNorm of q and k before RoPE (attention.py:83-95)."""
    qn = rms_norm(q.reshape(-1, head_dim), q_weight).view(q.shape)
    kn = rms_norm(k.reshape(-1, head_dim), k_weight).view(k.shape)
    return qn, kn


# ---------------------------------------------------------------------------
# Paged KV
# ---------------------------------------------------------------------------


def physical_pool(pages: torch.Tensor) -> torch.Tensor:
    """Physical [P, H, S, D] tensor behind a logical [P, H, D, S] pool.

    Zero-copy for KVPagedStorage.k_pages / v_pages; any other logical tensor is
    copied into the physical layout.
    """
    phys = pages.permute(0, 1, 3, 2)
    return phys if phys.is_contiguous() else phys.contiguous()


def _table_tensor(block_table: list[int], device: torch.device) -> torch.Tensor:
    return torch.tensor(block_table, dtype=torch.int32, device=device)


def gather_paged_kv(k_pages: torch.Tensor, v_pages: torch.Tensor, block_table: list[int],
                    page_size: int, num_tokens: int | None = None
                    ) -> tuple[torch.Tensor, torch.Tensor]:
    """Contiguous K, V of one request, each [1, num_tokens, n_kv_heads, head_dim]."""
    kp = physical_pool(k_pages)
    vp = physical_pool(v_pages)
    if kp.shape[2] != page_size:
        raise ValueError(f"page_size {page_size} does not match the pool ({kp.shape[2]})")
    n = len(block_table) * page_size if num_tokens is None else num_tokens
    if not block_table:
        n = 0
    bt = _table_tensor(block_table, kp.device)
    k = kernels.paged_kv_gather(kp, bt, n)
    v = kernels.paged_kv_gather(vp, bt, n)
    return k.unsqueeze(0), v.unsqueeze(0)


def paged_attention_v1(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor,
                       block_table: list[int], page_size: int, kv_num_tokens: int | None = None,
                       causal: bool = True) -> torch.Tensor:
    """Paged attention for one request; q [1, Sq, Hq, D] -> [1, Sq, Hq, D].

    Semantics of the reference (attention.py:151-190), including SDPA's top-left
    causal alignment: with causal=True a query at row i sees keys 0..i, so a single
    causal query sees only key 0. Decode callers pass causal=False
    (src/plastic_infer/exec/runner_paged.py:254-255). One query runs the paged decode
    kernel; several (prefill) run the tcgen05 paged prefill kernel straight from the pool
    when it covers the shape (bf16/f16, head_dim 64/128, pages of 16/32, G in 1/2/4/8/16).
    """
    n_kv = len(block_table) * page_size if kv_num_tokens is None else kv_num_tokens
    if not block_table:
        n_kv = 0
    B, Sq, Hq, D = q.shape
    if B != 1:
        raise ValueError("paged_attention_v1 takes one request (batch 1); use "
                         "kernels.paged_decode_attention for batches")
    if Sq == 1:
        kp = physical_pool(k_pages)
        vp = physical_pool(v_pages)
        ctx = min(1, n_kv) if causal else n_kv
        n_pages = -(-ctx // page_size) if ctx > 0 else 0
        bt = _table_tensor(block_table[:max(n_pages, 1)] if block_table else [0], kp.device)
        ctx_t = torch.tensor([ctx], dtype=torch.int32, device=kp.device)
        out = kernels.paged_decode_attention(q.reshape(1, Hq, D), kp, vp, bt.view(1, -1), ctx_t)
        return out.view(1, 1, Hq, D)
    # Prefill straight from the pool on the tcgen05 kernel (SDPA's top-left causal mask is
    # its causal mode with q_start 0); shapes it does not cover keep the reference algorithm
    # (gather, repeat_interleave, SDPA) over the kernel gather.
    kp = physical_pool(k_pages)
    if n_kv > 0 and kernels.prefill_supported(q, kp):
        vp = physical_pool(v_pages)
        n_pages = -(-n_kv // page_size)
        bt = _table_tensor(block_table[:n_pages], kp.device)
        return kernels.paged_prefill_attention(q, kp, vp, bt, n_kv, q_start=0, causal=causal,
                                               impl="tc")
    k, v = gather_paged_kv(k_pages, v_pages, block_table, page_size, n_kv)
    q_t = q.transpose(1, 2)
    k_t = k.transpose(1, 2)
    v_t = v.transpose(1, 2)
    Hkv = k_t.shape[1]
    if Hq != Hkv:
        assert Hq % Hkv == 0
        k_t = k_t.repeat_interleave(Hq // Hkv, dim=1)
        v_t = v_t.repeat_interleave(Hq // Hkv, dim=1)
    return F.scaled_dot_product_attention(q_t, k_t, v_t, is_causal=causal).transpose(1, 2)


def host_stream_attention_v1(q: torch.Tensor, host_chunks: list[tuple[torch.Tensor, torch.Tensor]],
                             resident_k: torch.Tensor, resident_v: torch.Tensor,
                             q_start_pos: int = 0, causal: bool = True) -> torch.Tensor:
    """Attention over host chunks ([H_kv, D, C] each, oldest first) plus a resident
    tail ([1, R, H_kv, D]); the reference's semantics (attention.py:193-250) computed by
    the flash-incremental kernel its docstring anticipates (pi_host_stream_attn).

    Nothing is concatenated: each chunk and the tail is one span of the kernel's KV
    sequence. Chunks in page-locked host memory (the host KV store's buffers) are read
    in place over the host link; pageable or other-dtype chunks are first copied to the
    query's GPU in q's dtype. Returns [1, q_len, Hq, D].
    """
    kernels._require_cuda(q)
    dev, dt = q.device, q.dtype

    def place(t: torch.Tensor) -> torch.Tensor:
        if t.dtype != dt or (t.is_cuda and t.device != dev) or (not t.is_cuda and not t.is_pinned()):
            return t.to(dev, dt)
        return t

    def pair(k: torch.Tensor, v: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        k, v = place(k), place(v)
        if k.stride() != v.stride():  # the kernel reads K and V of a span with one stride set
            k, v = k.to(dev).contiguous(), v.to(dev).contiguous()
        return k, v

    spans = []
    for kc, vc in host_chunks:
        kc, vc = pair(kc, vc)
        spans.append((kc.permute(0, 2, 1), vc.permute(0, 2, 1)))   # [H_kv, C, D]
    rk, rv = pair(resident_k[0], resident_v[0])                     # [R, H_kv, D]
    spans.append((rk.permute(1, 0, 2), rv.permute(1, 0, 2)))       # [H_kv, R, D]
    return kernels.host_stream_attention(q, spans, q_start=q_start_pos, causal=causal)
