"""The reference's CPU decode KV path, restated with the same PyTorch operations.

TEST INFRASTRUCTURE ONLY. This module is the timed reference arm of bench.py
(`--impl reference`) and is pinned by tests/test_oracle_golden.py against outputs of
the reference itself. The product path (plastic_infer_b200) never imports it.

plastic-infer's decode step (src/plastic_infer/exec/runner_paged.py:209-274) runs, per
request and layer:
  1. _write_kv_layer (runner_paged.py:112-129): the new token's K and V rows assigned
     into the logical pool [num_pages, kv_heads, head_dim, page_size] at
     (block_table[layer][pos // S], :, :, pos % S);
  2. _attn_paged(..., causal=False) (runner_paged.py:253-254, 36-59), which is
     paged_attention_v1 (src/plastic_infer/exec/attention.py:151-190): gather_paged_kv
     (index_select of the request's pages, permute, reshape, trim; attention.py:103-148),
     a repeat_interleave of the KV heads to the query heads, and
     torch.nn.functional.scaled_dot_product_attention.
The reference repository is not present on the machine that runs the benchmark, so the
same operations are written out here, in the same order and on the same dtypes, so that
the timed CPU work is the reference's own algorithm. The numpy oracle
(paged_kv_oracle.py) remains the parity checker.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def write_kv_token(k_pages: torch.Tensor, v_pages: torch.Tensor, page: int, offset: int,
                   k_row: torch.Tensor, v_row: torch.Tensor) -> None:
    """pool[page, :, :, offset] = row for K and V (runner_paged.py:128-129)."""
    k_pages[page, :, :, offset] = k_row
    v_pages[page, :, :, offset] = v_row


def gather_pages(k_pages: torch.Tensor, v_pages: torch.Tensor, pages: list[int], page_size: int,
                 num_tokens: int) -> tuple[torch.Tensor, torch.Tensor]:
    """[1, num_tokens, kv_heads, head_dim] K and V of one request (attention.py:133-148)."""
    ids = torch.tensor(pages, dtype=torch.long, device=k_pages.device)
    kg = k_pages.index_select(0, ids)
    vg = v_pages.index_select(0, ids)
    n, h, d, _ = kg.shape
    k = kg.permute(0, 3, 1, 2).reshape(n * page_size, h, d)[:num_tokens]
    v = vg.permute(0, 3, 1, 2).reshape(n * page_size, h, d)[:num_tokens]
    return k.unsqueeze(0), v.unsqueeze(0)


def decode_attention(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor,
                     pages: list[int], page_size: int, num_tokens: int) -> torch.Tensor:
    """paged_attention_v1 for one request with causal=False: q [1, 1, Hq, D] -> [1, 1, Hq, D]."""
    if num_tokens <= 0:
        return torch.zeros_like(q)  # SDPA over zero keys (attention.py:127-131 returns empty K/V)
    k, v = gather_pages(k_pages, v_pages, pages, page_size, num_tokens)
    q_t, k_t, v_t = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    groups = q_t.shape[1] // k_t.shape[1]
    if groups != 1:
        k_t = k_t.repeat_interleave(groups, dim=1)
        v_t = v_t.repeat_interleave(groups, dim=1)
    return F.scaled_dot_product_attention(q_t, k_t, v_t, is_causal=False).transpose(1, 2)


def decode_layer(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                 k_pages: torch.Tensor, v_pages: torch.Tensor, tables: list[list[int]],
                 ctx_lens: list[int], page_size: int) -> torch.Tensor:
    """One layer of a decode step for a batch, one request after another as the
    reference's runner does: write request b's new row at position ctx_lens[b] - 1, then
    attend its first ctx_lens[b] tokens. q [B, Hq, D], k_new/v_new [B, Hkv, D]."""
    out = torch.empty_like(q)
    for b, n in enumerate(ctx_lens):
        n = int(n)
        if n > 0:
            pos = n - 1
            write_kv_token(k_pages, v_pages, tables[b][pos // page_size], pos % page_size,
                           k_new[b], v_new[b])
        npg = -(-n // page_size)
        out[b] = decode_attention(q[b].view(1, 1, *q.shape[1:]), k_pages, v_pages,
                                  tables[b][:npg], page_size, n).view(q.shape[1:])
    return out
