"""Tensor-level wrappers over the C ABI (the batched entry points of the hot path).

These are the batched additions behind the reference's single-request API:

  kv_index_copy          one launch writes a whole step's new K/V rows
                         (reference: _write_kv_layer, src/plastic_infer/exec/runner_paged.py:112-129)
  paged_decode_attention one launch attends every request of the batch
                         (reference: paged_attention_v1, src/plastic_infer/exec/attention.py:151-190)
  paged_kv_gather        contiguous gather of one request
                         (reference: gather_paged_kv, src/plastic_infer/exec/attention.py:103-148)
  page_gather / page_scatter
                         pool <-> staging moves for the host store
                         (reference: src/plastic_infer/kv/kv_store.py:258-269, 311-321)
  paged_decode_attention_gather
                         decode attention of one KV-head shard with the all-gather of the
                         per-rank outputs fused in (NVLink peer stores; multi-GPU)
  decode_prologue        QK-norm + RoPE of a step's q/k rows and the K/V slot write, one
                         launch (reference: attention.py:23-95 + _write_kv_layer)
  paged_prefill_attention
                         one request's prefill straight from the pool
                         (reference: _attn_paged, src/plastic_infer/exec/runner_paged.py:36-95)
  expert_slot_copy       MoE expert rows from pinned host banks into device slots, all banks
                         in one launch (reference: fast_index_copy_multi_jit)
  host_stream_attention  one request's attention over host-resident chunks (pinned, read in
                         place) plus a device tail (reference: host_stream_attention_v1,
                         src/plastic_infer/exec/attention.py:193-250)
  set_programmatic_launch
                         programmatic dependent launch for the index-copy, prologue and
                         attention kernels
  set_decode_attn_ring   page-ring depth of plain attention launches (automatic, deep or
                         shallow), so either kernel instance can be run at any size

Pools are the *physical* tensors [num_pages, kv_heads, page_size, head_dim]. Every
function launches on torch's current stream, as the reference's ctypes launch does
(src/plastic_infer/kernel/fast_index_copy.py:185), and raises `KernelError` on a
non-zero status. Inputs must be CUDA tensors (host_stream_attention also reads
page-locked host tensors in place); there is no CPU path.
"""

from __future__ import annotations

import ctypes
import math
import threading

import numpy as np
import torch

from . import _capi

_DTYPES = {
    torch.float32: _capi.PI_DTYPE_F32,
    torch.bfloat16: _capi.PI_DTYPE_BF16,
    torch.float16: _capi.PI_DTYPE_F16,
}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPES[dt]
    except KeyError:
        raise TypeError(f"unsupported KV dtype {dt}; expected float32, bfloat16 or float16")


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise ValueError(
                "plastic_infer_b200 kernels need CUDA tensors (no CPU fallback); got "
                f"{t.device}"
            )


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _err_ptr(err: torch.Tensor | None) -> int | None:
    if err is None:
        return None
    if err.dtype != torch.int32 or not err.is_cuda or err.numel() < 1:
        raise ValueError("err must be a CUDA int32 tensor with at least one element")
    return err.data_ptr()


def _check_pool(pool: torch.Tensor, name: str) -> tuple[int, int, int, int]:
    if pool.dim() != 4 or not pool.is_contiguous():
        raise ValueError(f"{name} must be a contiguous [num_pages, kv_heads, page_size, head_dim] tensor")
    return tuple(pool.shape)  # type: ignore[return-value]


# ---------------------------------------------------------------------------
# a1: slot-mapping index-copy
# ---------------------------------------------------------------------------


def kv_index_copy(
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    k_new: torch.Tensor,
    v_new: torch.Tensor,
    slot_mapping: torch.Tensor,
    err: torch.Tensor | None = None,
) -> None:
    """pool[slot // S, :, slot % S, :] = new[i] for every i with slot_mapping[i] >= 0.

    k_new / v_new: [n, kv_heads, head_dim] (any token stride, heads contiguous) or
    [1, n, kv_heads, head_dim] as produced by the reference runner.
    slot_mapping: int64 [n] on the pool's device; slot = page_id * page_size + offset.
    """
    P, H, S, D = _check_pool(k_pool, "k_pool")
    if v_pool.shape != k_pool.shape or v_pool.dtype != k_pool.dtype:
        raise ValueError("k_pool and v_pool must have the same shape and dtype")
    if k_new.dim() == 4:
        k_new = k_new.reshape(-1, k_new.shape[-2], k_new.shape[-1])
        v_new = v_new.reshape(-1, v_new.shape[-2], v_new.shape[-1])
    if k_new.shape != v_new.shape or tuple(k_new.shape[1:]) != (H, D):
        raise ValueError(f"k_new/v_new must be [n, {H}, {D}], got {tuple(k_new.shape)}")
    if k_new.dtype != k_pool.dtype or v_new.dtype != k_pool.dtype:
        raise TypeError("new K/V rows must have the pool dtype")
    n = k_new.shape[0]
    if slot_mapping.dtype != torch.int64 or slot_mapping.shape != (n,):
        raise ValueError("slot_mapping must be int64 of shape [n]")
    _require_cuda(k_pool, v_pool, k_new, v_new, slot_mapping)
    if n == 0:
        return
    # Rows of one token must be [H, D] contiguous and K/V must share one token
    # stride; tokens themselves may be strided (e.g. slices of a fused QKV output).
    if not (k_new.stride(2) == 1 and k_new.stride(1) == D and v_new.stride() == k_new.stride()):
        k_new = k_new.contiguous()
        v_new = v_new.contiguous()
    slot_mapping = slot_mapping.contiguous()
    _capi.call(
        "pi_kv_index_copy",
        k_pool.data_ptr(), v_pool.data_ptr(), k_new.data_ptr(), v_new.data_ptr(),
        slot_mapping.data_ptr(), n, H, D, S, P * S, dtype_code(k_pool.dtype), k_new.stride(0),
        _err_ptr(err), _stream(),
    )


# ---------------------------------------------------------------------------
# f1: fused decode prologue (QK-norm + RoPE + slot-mapping write)
# ---------------------------------------------------------------------------


def rope_inv_freq(head_dim: int, base: float, device: torch.device | str = "cpu") -> torch.Tensor:
    """fp32 [head_dim / 2] rotary frequencies 1 / base^(2j / head_dim).

    Computed on the CPU with the expression of build_rope_cache's fp32 table
    (src/plastic_infer/exec/attention.py:68), so pos * inv_freq[j] is exactly the angle
    that table holds at (pos, j); then moved to `device`.
    """
    inv = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    return inv.to(device)


def decode_prologue(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    positions: torch.Tensor,
    inv_freq: torch.Tensor,
    slot_mapping: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    q_norm_weight: torch.Tensor | None = None,
    k_norm_weight: torch.Tensor | None = None,
    eps: float = 1e-5,
    q_out: torch.Tensor | None = None,
    err: torch.Tensor | None = None,
) -> torch.Tensor:
    """One launch per layer: QK-norm (optional) + RoPE of the step's q and k rows, and the
    write of the new K/V rows at their slots (the kv_index_copy semantics).

    q [B, Hq, D], k / v [B, Hkv, D]: the projection outputs (heads contiguous; any request
    stride, k and v sharing one, e.g. slices of a fused QKV output). positions int64
    [B]: each request's new-token position. inv_freq fp32 [D/2] (rope_inv_freq).
    slot_mapping int64 [B] (< 0: no K/V row). Returns q_out [B, Hq, D] in the pool dtype.
    Replaces qk_norm + rope_positions + _write_kv_layer of the reference runners
    (src/plastic_infer/exec/attention.py:23-95, src/plastic_infer/exec/runner_paged.py:112-129).
    """
    P, Hkv, S, D = _check_pool(k_pool, "k_pool")
    if v_pool.shape != k_pool.shape or v_pool.dtype != k_pool.dtype:
        raise ValueError("k_pool and v_pool must have the same shape and dtype")
    B, Hq = q.shape[0], q.shape[1]
    if q.dim() != 3 or q.shape[2] != D or tuple(k.shape) != (B, Hkv, D) or k.shape != v.shape:
        raise ValueError(f"q must be [B, Hq, {D}] and k, v [B, {Hkv}, {D}]")
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError("q, k and v must share one dtype")
    for t, name in ((q, "q"), (k, "k"), (v, "v")):
        if t.stride(2) != 1 or t.stride(1) != D:
            raise ValueError(f"{name}: heads must be contiguous rows of head_dim elements")
    if k.stride(0) != v.stride(0):
        raise ValueError("k and v must share one request stride")
    if positions.dtype != torch.int64 or positions.shape != (B,):
        raise ValueError("positions must be int64 [B]")
    if slot_mapping.dtype != torch.int64 or slot_mapping.shape != (B,):
        raise ValueError("slot_mapping must be int64 [B]")
    if inv_freq.dtype != torch.float32 or inv_freq.numel() != D // 2:
        raise ValueError(f"inv_freq must be float32 [{D // 2}]")
    if (q_norm_weight is None) != (k_norm_weight is None):
        raise ValueError("give both QK-norm weights or neither")
    _require_cuda(q, k, v, positions, inv_freq, slot_mapping, k_pool, v_pool)
    if q_out is None:
        q_out = torch.empty((B, Hq, D), dtype=k_pool.dtype, device=q.device)
    elif q_out.dtype != k_pool.dtype or tuple(q_out.shape) != (B, Hq, D) or q_out.stride(2) != 1 \
            or q_out.stride(1) != D:
        raise ValueError("q_out must be [B, Hq, D] in the pool dtype with contiguous heads")
    qw = kw = None
    if q_norm_weight is not None:
        qw = q_norm_weight.to(q.dtype).contiguous()
        kw = k_norm_weight.to(q.dtype).contiguous()
        if qw.numel() != D or kw.numel() != D:
            raise ValueError(f"QK-norm weights must have {D} elements")
    positions = positions.contiguous()
    slot_mapping = slot_mapping.contiguous()
    inv_freq = inv_freq.contiguous()
    _capi.call(
        "pi_decode_prologue",
        q_out.data_ptr(), q_out.stride(0), k_pool.data_ptr(), v_pool.data_ptr(),
        q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), k.stride(0), dtype_code(q.dtype),
        qw.data_ptr() if qw is not None else None, kw.data_ptr() if kw is not None else None,
        float(eps), inv_freq.data_ptr(), positions.data_ptr(), slot_mapping.data_ptr(),
        B, Hq, Hkv, D, S, P * S, dtype_code(k_pool.dtype), _err_ptr(err), _stream(),
    )
    return q_out


# ---------------------------------------------------------------------------
# f4: MoE expert-slot copy (all banks, one launch)
# ---------------------------------------------------------------------------


def expert_slot_copy(
    dst_ptrs: torch.Tensor,
    src_ptrs: torch.Tensor,
    feat_bytes: torch.Tensor,
    dst_indices: torch.Tensor,
    src_indices: torch.Tensor,
    num_indices: torch.Tensor | None = None,
    err: torch.Tensor | None = None,
) -> None:
    """dst_b[dst_indices[i]] = src_b[src_indices[i]] for every bank b and i < n, one launch.

    The signature of the reference's fast_index_copy_multi_jit
    (src/plastic_infer/kernel/fast_index_copy.py:208-244): dst_ptrs / src_ptrs / feat_bytes
    are int64 [num_banks] CUDA tensors (slot-cache base, host-bank device alias, row
    bytes), the index tensors int32 or int64 CUDA [L], num_indices an optional CUDA
    int64 [1] valid length (n = min(num_indices[0], L)).
    """
    for t, name in ((dst_ptrs, "dst_ptrs"), (src_ptrs, "src_ptrs"), (feat_bytes, "feat_bytes")):
        if t.dtype != torch.int64 or t.dim() != 1:
            raise ValueError(f"{name} must be an int64 [num_banks] tensor")
    if not (dst_ptrs.numel() == src_ptrs.numel() == feat_bytes.numel()):
        raise ValueError("dst_ptrs, src_ptrs and feat_bytes must have one entry per bank")
    if dst_indices.shape != src_indices.shape or dst_indices.dtype != src_indices.dtype \
            or dst_indices.dtype not in (torch.int32, torch.int64) or dst_indices.dim() != 1:
        raise ValueError("dst_indices and src_indices must be matching int32/int64 [L] tensors")
    if num_indices is not None and (num_indices.dtype != torch.int64 or num_indices.numel() < 1):
        raise ValueError("num_indices must be an int64 [1] tensor")
    tensors = [dst_ptrs, src_ptrs, feat_bytes, dst_indices, src_indices]
    if num_indices is not None:
        tensors.append(num_indices)
    _require_cuda(*tensors)
    _capi.call(
        "pi_expert_slot_copy",
        dst_ptrs.contiguous().data_ptr(), src_ptrs.contiguous().data_ptr(),
        feat_bytes.contiguous().data_ptr(), dst_ptrs.numel(), dst_indices.contiguous().data_ptr(),
        src_indices.contiguous().data_ptr(), dst_indices.numel(),
        num_indices.data_ptr() if num_indices is not None else None,
        1 if dst_indices.dtype == torch.int32 else 0, _err_ptr(err), _stream(),
    )


# ---------------------------------------------------------------------------
# a2: paged decode attention
# ---------------------------------------------------------------------------


class Workspace:
    """Zero-initialised device scratch for pi_paged_decode_attn, grown on demand.

    The kernel leaves its counter region zero on exit, so the buffer is zeroed once
    at allocation. Launches that share one Workspace must be ordered (same stream);
    give concurrent streams their own Workspace.
    """

    def __init__(self, device: torch.device) -> None:
        self.device = torch.device(device)
        self.buf: torch.Tensor | None = None

    def get(self, nbytes: int) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes:
            n = max(nbytes, 1 << 20)
            self.buf = torch.zeros(n, dtype=torch.uint8, device=self.device)
        return self.buf


_ws_lock = threading.Lock()
_default_ws: dict[int, Workspace] = {}


def default_workspace(device: torch.device) -> Workspace:
    idx = torch.device(device).index
    if idx is None:
        idx = torch.cuda.current_device()
    with _ws_lock:
        ws = _default_ws.get(idx)
        if ws is None:
            ws = _default_ws[idx] = Workspace(torch.device("cuda", idx))
        return ws


def set_programmatic_launch(enable: bool) -> None:
    """Programmatic dependent launch for every later index-copy and attention launch.

    When on, a kernel may launch while the previous kernel on its stream is still
    running: the attention computes its work split and fetches its first page ids
    (reading only ctx_lens and block_tables) before it waits for that kernel. So the
    kernel launched just before an attention must not write its ctx_lens or
    block_tables. Off by default.
    """
    _capi.call("pi_set_programmatic_launch", 1 if enable else 0)


_RING_MODES = {"auto": _capi.PI_ATTN_RING_AUTO, "deep": _capi.PI_ATTN_RING_DEEP,
               "shallow": _capi.PI_ATTN_RING_SHALLOW}


def set_decode_attn_ring(mode: str) -> None:
    """Page-ring depth of every later plain paged_decode_attention launch.

    "auto" (the default) picks per launch: a two-stage ring with two CTAs per SM when
    batch x block-table width x KV heads is large, else a deep ring (4 stages at
    head_dim <= 128) with one CTA per SM. "deep" and "shallow" force one of them
    (shallow only where two CTAs fit on an SM). Launches with the fused append or the
    peer all-gather always use the deep ring.
    """
    try:
        code = _RING_MODES[mode]
    except KeyError:
        raise ValueError(f"ring mode must be one of {sorted(_RING_MODES)}, got {mode!r}")
    _capi.call("pi_set_decode_attn_ring", code)


def decode_attn_ring_stages(batch: int, bt_stride: int, num_q_heads: int, num_kv_heads: int,
                            head_dim: int, page_size: int, num_pages: int,
                            dtype: torch.dtype) -> int:
    """Ring stages a plain attention launch of this shape would use now (0: SIMT path)."""
    return int(_capi.load().pi_paged_decode_attn_ring_stages(
        batch, bt_stride, num_q_heads, num_kv_heads, head_dim, page_size, num_pages,
        dtype_code(dtype)))


def workspace_bytes(batch: int, num_q_heads: int, num_kv_heads: int, head_dim: int) -> int:
    return int(_capi.load().pi_paged_decode_attn_workspace_bytes(batch, num_q_heads, num_kv_heads, head_dim))


def paged_decode_attention(
    q: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_tables: torch.Tensor,
    ctx_lens: torch.Tensor,
    scale: float | None = None,
    out: torch.Tensor | None = None,
    workspace: Workspace | None = None,
    err: torch.Tensor | None = None,
    k_new: torch.Tensor | None = None,
    v_new: torch.Tensor | None = None,
    slot_mapping: torch.Tensor | None = None,
) -> torch.Tensor:
    """Decode attention of q [B, Hq, D] over each request's first ctx_lens[b] tokens.

    block_tables: int32 [B, max_pages] page ids; ctx_lens: int32 [B]. Returns
    out [B, Hq, D] in the pool dtype (fp32 softmax/accumulation inside).

    With k_new / v_new [B, Hkv, D] and slot_mapping int64 [B], the step's new rows
    are first written at their slots (the kv_index_copy semantics) in the same
    launch: a whole decode layer's KV path is then one kernel.
    """
    P, Hkv, S, D = _check_pool(k_pool, "k_pool")
    if v_pool.shape != k_pool.shape or v_pool.dtype != k_pool.dtype:
        raise ValueError("k_pool and v_pool must have the same shape and dtype")
    if q.dim() != 3 or q.shape[2] != D:
        raise ValueError(f"q must be [B, Hq, {D}], got {tuple(q.shape)}")
    B, Hq, _ = q.shape
    if Hq % Hkv != 0:
        raise ValueError(f"num_q_heads {Hq} not a multiple of num_kv_heads {Hkv}")
    if q.dtype != k_pool.dtype:
        raise TypeError("q must have the pool dtype")
    if block_tables.dtype != torch.int32 or block_tables.dim() != 2 or block_tables.shape[0] != B:
        raise ValueError("block_tables must be int32 [B, max_pages]")
    if ctx_lens.dtype != torch.int32 or ctx_lens.shape != (B,):
        raise ValueError("ctx_lens must be int32 [B]")
    _require_cuda(q, k_pool, v_pool, block_tables, ctx_lens)
    if q.stride(2) != 1 or q.stride(1) != D:
        q = q.contiguous()
    if block_tables.stride(1) != 1:
        block_tables = block_tables.contiguous()
    ctx_lens = ctx_lens.contiguous()
    if out is None:
        out = torch.empty((B, Hq, D), dtype=q.dtype, device=q.device)
    elif out.shape != (B, Hq, D) or out.dtype != q.dtype or out.stride(2) != 1 or out.stride(1) != D:
        raise ValueError("out must be [B, Hq, D] with contiguous heads, pool dtype")
    if B == 0:
        return out
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    nbytes = workspace_bytes(B, Hq, Hkv, D)
    ws = (workspace or default_workspace(q.device)).get(nbytes)
    if k_new is None and v_new is None and slot_mapping is None:
        _capi.call(
            "pi_paged_decode_attn",
            out.data_ptr(), q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(),
            block_tables.data_ptr(), block_tables.stride(0), ctx_lens.data_ptr(),
            B, Hq, Hkv, D, S, P, float(scale), dtype_code(q.dtype), q.stride(0), out.stride(0),
            ws.data_ptr(), ws.numel(), _err_ptr(err), _stream(),
        )
        return out
    # Fused append: write one new K/V row per request, then attend (one launch).
    if k_new is None or v_new is None or slot_mapping is None:
        raise ValueError("k_new, v_new and slot_mapping go together")
    if k_new.shape != (B, Hkv, D) or v_new.shape != (B, Hkv, D):
        raise ValueError(f"k_new/v_new must be [{B}, {Hkv}, {D}]")
    if k_new.dtype != k_pool.dtype or v_new.dtype != k_pool.dtype:
        raise TypeError("new K/V rows must have the pool dtype")
    if slot_mapping.dtype != torch.int64 or slot_mapping.shape != (B,):
        raise ValueError("slot_mapping must be int64 [B]")
    _require_cuda(k_new, v_new, slot_mapping)
    if not (k_new.stride(2) == 1 and k_new.stride(1) == D and v_new.stride() == k_new.stride()):
        k_new = k_new.contiguous()
        v_new = v_new.contiguous()
    slot_mapping = slot_mapping.contiguous()
    _capi.call(
        "pi_paged_decode_attn_append",
        out.data_ptr(), q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), k_new.data_ptr(),
        v_new.data_ptr(), slot_mapping.data_ptr(), k_new.stride(0),
        block_tables.data_ptr(), block_tables.stride(0), ctx_lens.data_ptr(),
        B, Hq, Hkv, D, S, P, float(scale), dtype_code(q.dtype), q.stride(0), out.stride(0),
        ws.data_ptr(), ws.numel(), _err_ptr(err), _stream(),
    )
    return out


# ---------------------------------------------------------------------------
# gather_paged_kv and a3: page moves
# ---------------------------------------------------------------------------


def paged_kv_gather(pool: torch.Tensor, block_table: torch.Tensor, num_tokens: int,
                    err: torch.Tensor | None = None) -> torch.Tensor:
    """out[t, h, :] = pool[block_table[t // S], h, t % S, :] -> [num_tokens, H, D]."""
    P, H, S, D = _check_pool(pool, "pool")
    if block_table.dtype != torch.int32 or block_table.dim() != 1:
        raise ValueError("block_table must be int32 [n_pages]")
    if num_tokens > block_table.numel() * S:
        raise ValueError("num_tokens exceeds the block table's pages")
    _require_cuda(pool, block_table)
    out = torch.empty((num_tokens, H, D), dtype=pool.dtype, device=pool.device)
    if num_tokens == 0:
        return out
    _capi.call(
        "pi_paged_kv_gather",
        out.data_ptr(), pool.data_ptr(), block_table.contiguous().data_ptr(), num_tokens, H, D, S,
        P, dtype_code(pool.dtype), _err_ptr(err), _stream(),
    )
    return out


def _page_move(func: str, pool: torch.Tensor, staging: torch.Tensor, page_ids: torch.Tensor,
               pages_per_group: int, err: torch.Tensor | None) -> None:
    P, H, S, D = _check_pool(pool, "pool")
    if page_ids.dtype != torch.int32 or page_ids.dim() != 1:
        raise ValueError("page_ids must be int32 [n]")
    n = page_ids.numel()
    tile_bytes = S * D * pool.element_size()
    if not staging.is_contiguous() or staging.numel() * staging.element_size() < n * H * tile_bytes:
        raise ValueError("staging must be contiguous and hold n * kv_heads * page_size * head_dim elements")
    if pages_per_group <= 0 or n % pages_per_group != 0:
        raise ValueError("page count must be a multiple of pages_per_group")
    _require_cuda(pool, staging, page_ids)
    if n == 0:
        return
    page_ids = page_ids.contiguous()
    if func == "pi_page_gather":
        args = (staging.data_ptr(), pool.data_ptr())
    else:
        args = (pool.data_ptr(), staging.data_ptr())
    _capi.call(func, *args, page_ids.data_ptr(), n, H, tile_bytes, pages_per_group, P,
               _err_ptr(err), _stream())


def page_gather(pool: torch.Tensor, page_ids: torch.Tensor, staging: torch.Tensor,
                pages_per_group: int = 1, err: torch.Tensor | None = None) -> None:
    """staging <- pool pages, grouped head-major (see include/plastic_kv.h)."""
    _page_move("pi_page_gather", pool, staging, page_ids, pages_per_group, err)


def page_scatter(staging: torch.Tensor, page_ids: torch.Tensor, pool: torch.Tensor,
                 pages_per_group: int = 1, err: torch.Tensor | None = None) -> None:
    """pool pages <- staging (inverse of page_gather)."""
    _page_move("pi_page_scatter", pool, staging, page_ids, pages_per_group, err)


# ---------------------------------------------------------------------------
# f3: paged prefill attention
# ---------------------------------------------------------------------------

PREFILL_GROUPS = (1, 2, 4, 8, 16)


def prefill_supported(q: torch.Tensor, k_pool: torch.Tensor) -> bool:
    """Whether pi_paged_prefill_attn covers this q / pool combination."""
    if k_pool.dim() != 4 or q.dim() not in (3, 4):
        return False
    P, Hkv, S, D = k_pool.shape
    Hq = q.shape[-2]
    return (k_pool.dtype in (torch.bfloat16, torch.float16) and q.dtype == k_pool.dtype
            and D in (64, 128) and S in (16, 32) and q.shape[-1] == D and Hq % Hkv == 0
            and Hq // Hkv in PREFILL_GROUPS)


def paged_prefill_attention(
    q: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_table: torch.Tensor,
    kv_len: int,
    q_start: int = 0,
    causal: bool = True,
    scale: float | None = None,
    out: torch.Tensor | None = None,
    err: torch.Tensor | None = None,
    impl: str = "mma",
) -> torch.Tensor:
    """Prefill attention of one request's q [q_len, Hq, D] (or [1, q_len, Hq, D]) over the
    first kv_len tokens of its pages (block_table: int32 [n] page ids, device).

    Query i sits at position q_start + i; with `causal` it sees keys j <= q_start + i
    (the reference's is_causal when q_start == 0, its offset mask otherwise:
    src/plastic_infer/exec/runner_paged.py:36-95). Returns [q_len, Hq, D] in the pool dtype
    (the input's leading batch axis is kept when given). `impl` picks the kernel: "tc"
    (tcgen05, S and O in tensor memory) or "mma" (mma.sync, accumulators in registers).
    """
    if impl not in ("tc", "mma"):
        raise ValueError(f"impl must be 'tc' or 'mma', got {impl!r}")
    P, Hkv, S, D = _check_pool(k_pool, "k_pool")
    if v_pool.shape != k_pool.shape or v_pool.dtype != k_pool.dtype:
        raise ValueError("k_pool and v_pool must have the same shape and dtype")
    batched = q.dim() == 4
    if batched:
        if q.shape[0] != 1:
            raise ValueError("prefill attends one request: q must be [1, q_len, Hq, D]")
        q3 = q[0]
    else:
        q3 = q
    if q3.dim() != 3 or q3.shape[2] != D:
        raise ValueError(f"q must be [q_len, Hq, {D}]")
    if not prefill_supported(q3, k_pool):
        raise ValueError("shape or dtype not covered by the prefill kernel (bf16/f16, head_dim "
                         "64/128, page 16/32, Hq/Hkv in 1/2/4/8/16)")
    if block_table.dtype != torch.int32 or block_table.dim() != 1:
        raise ValueError("block_table must be int32 [n]")
    q_len, Hq = q3.shape[0], q3.shape[1]
    if kv_len > block_table.numel() * S or kv_len < 0 or q_start < 0:
        raise ValueError("kv_len must be within the block table's pages")
    _require_cuda(q3, k_pool, v_pool, block_table)
    if q3.stride(2) != 1 or q3.stride(1) != D:
        q3 = q3.contiguous()
    if out is None:
        out3 = torch.empty((q_len, Hq, D), dtype=k_pool.dtype, device=q3.device)
    else:
        out3 = out[0] if out.dim() == 4 else out
        if out3.shape != (q_len, Hq, D) or out3.dtype != k_pool.dtype or out3.stride(2) != 1 \
                or out3.stride(1) != D:
            raise ValueError("out must be [q_len, Hq, D] in the pool dtype with contiguous heads")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    block_table = block_table.contiguous()
    dst = out3
    if impl == "tc":
        # the tcgen05 kernel moves q and the output by TMA: 16-byte aligned rows
        if q3.data_ptr() % 16 or q3.stride(0) % 8:
            q3 = q3.clone(memory_format=torch.contiguous_format)
        if dst.data_ptr() % 16 or dst.stride(0) % 8:
            dst = torch.empty((q_len, Hq, D), dtype=k_pool.dtype, device=q3.device)
    _capi.call(
        "pi_paged_prefill_attn_tc" if impl == "tc" else "pi_paged_prefill_attn",
        dst.data_ptr(), q3.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(),
        block_table.data_ptr(), block_table.numel(), q_len, int(kv_len), int(q_start),
        1 if causal else 0, Hq, Hkv, D, S, P, float(scale), dtype_code(k_pool.dtype),
        q3.stride(0), dst.stride(0), _err_ptr(err), _stream(),
    )
    if dst is not out3:
        out3.copy_(dst)
    if out is not None:
        return out
    return out3.unsqueeze(0) if batched else out3


# ---------------------------------------------------------------------------
# f2: attention over host-resident chunks + a device tail, read in place
# ---------------------------------------------------------------------------

_keep_lock = threading.Lock()
_keep: list[tuple[torch.cuda.Event, tuple]] = []
_hs_ws: dict[int, Workspace] = {}


def _keep_until_done(tensors: list[torch.Tensor]) -> None:
    """Hold host tensors a launch reads in place until the launch has run: torch cannot
    see a kernel's reads of pinned memory, and would otherwise recycle the pages."""
    if not tensors or torch.cuda.is_current_stream_capturing():
        return
    ev = torch.cuda.Event()
    ev.record()
    with _keep_lock:
        _keep[:] = [(e, t) for e, t in _keep if not e.query()]
        _keep.append((ev, tuple(tensors)))


def host_stream_attention(
    q: torch.Tensor,
    kv_spans,
    q_start: int = 0,
    causal: bool = True,
    scale: float | None = None,
    out: torch.Tensor | None = None,
    workspace: Workspace | None = None,
    err: torch.Tensor | None = None,
    num_kv_heads: int | None = None,
) -> torch.Tensor:
    """Attention of one request over a KV sequence given as spans, on the host or the GPU.

    q is [q_len, Hq, D] (or [1, q_len, Hq, D]) on the GPU; query i sits at position
    q_start + i. kv_spans is a sequence of (k, v) views shaped [H_kv, T, D] (any strides;
    k and v alike) that concatenate, in order, into the request's keys and values. A span
    lives on the query's GPU or in page-locked host memory, which the kernel reads in
    place over the host link: host chunks are never staged or materialised. With
    `causal`, query i sees keys j <= q_start + i; otherwise every key. Returns
    [q_len, Hq, D] in q's dtype (the leading batch axis is kept when given).

    The pinned spans stay referenced until the launch has run. Under CUDA-graph capture
    the caller keeps them alive for the graph's lifetime.
    """
    batched = q.dim() == 4
    if batched:
        if q.shape[0] != 1:
            raise ValueError("host-stream attention attends one request: q must be [1, q_len, Hq, D]")
        q3 = q[0]
    else:
        q3 = q
    if q3.dim() != 3:
        raise ValueError("q must be [q_len, Hq, D]")
    _require_cuda(q3)
    q_len, Hq, D = q3.shape
    if q_start < 0:
        raise ValueError("q_start must be >= 0")
    if q3.stride(2) != 1 or q3.stride(1) != D:
        q3 = q3.contiguous()
    code = dtype_code(q3.dtype)
    kv_spans = list(kv_spans)
    if len(kv_spans) > _capi.HS_MAX_SPANS:
        raise ValueError(f"at most {_capi.HS_MAX_SPANS} spans per call")
    rows: list[tuple[int, int, int, int, int, int]] = []
    hkv = num_kv_heads
    kv_len = 0
    host: list[torch.Tensor] = []
    for i, (k, v) in enumerate(kv_spans):
        if k.dim() != 3 or k.shape != v.shape or k.stride() != v.stride():
            raise ValueError("each span is a (k, v) pair of [H_kv, T, D] views with equal strides")
        if k.shape[2] != D:
            raise ValueError(f"span {i} has head_dim {k.shape[2]}, q has {D}")
        if hkv is None:
            hkv = k.shape[0]
        elif k.shape[0] != hkv:
            raise ValueError("every span must have the same number of KV heads")
        if k.dtype != q3.dtype or v.dtype != q3.dtype:
            raise TypeError(f"span {i} is {k.dtype}; q is {q3.dtype}")
        if k.is_cuda or v.is_cuda:
            if k.device != q3.device or v.device != q3.device:
                raise ValueError(f"span {i} is on {k.device}, q on {q3.device}")
        else:
            if not (k.is_pinned() and v.is_pinned()):
                raise ValueError(f"host span {i} must be in page-locked memory (Tensor.pin_memory())")
            host += [k, v]
        rows.append((k.data_ptr(), v.data_ptr(), k.shape[1], k.stride(0), k.stride(1), k.stride(2)))
        kv_len += k.shape[1]
    if hkv is None:
        hkv = Hq  # no keys at all: every row is zero
    if Hq % hkv:
        raise ValueError(f"Hq={Hq} is not a multiple of H_kv={hkv}")
    if out is None:
        out3 = torch.empty((q_len, Hq, D), dtype=q3.dtype, device=q3.device)
    else:
        out3 = out[0] if out.dim() == 4 else out
        if out3.shape != (q_len, Hq, D) or out3.dtype != q3.dtype or out3.stride(2) != 1 \
                or out3.stride(1) != D:
            raise ValueError("out must be [q_len, Hq, D] in q's dtype with contiguous heads")
    # pi_kv_span_t[]: six 64-bit fields per span (two addresses, length, three strides)
    table = np.array(rows if rows else [(0, 0, 0, 0, 0, 1)], dtype=np.uint64)
    _host_stream_launch(q3, out3, table, len(kv_spans), hkv, kv_len, q_start, causal, scale,
                        workspace, err)
    _keep_until_done(host)
    if out is not None:
        return out
    return out3.unsqueeze(0) if batched else out3


def _host_stream_launch(q3: torch.Tensor, out3: torch.Tensor, table: np.ndarray, n_spans: int,
                        hkv: int, kv_len: int, q_start: int, causal: bool, scale: float | None,
                        workspace: Workspace | None, err: torch.Tensor | None) -> None:
    q_len, Hq, D = q3.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    nbytes = int(_capi.load().pi_host_stream_attn_workspace_size(q_len, Hq, hkv, D, kv_len))
    ws_ptr = None
    if nbytes:
        if workspace is None:
            idx = q3.device.index
            with _ws_lock:
                workspace = _hs_ws.get(idx)
                if workspace is None:
                    workspace = _hs_ws[idx] = Workspace(q3.device)
        ws_ptr = workspace.get(nbytes).data_ptr()
    _capi.call(
        "pi_host_stream_attn",
        out3.data_ptr(), q3.data_ptr(), q3.stride(0), out3.stride(0), table.ctypes.data,
        n_spans, q_len, int(q_start), 1 if causal else 0, Hq, hkv, D, float(scale),
        dtype_code(q3.dtype), ws_ptr, nbytes, _capi.HS_SPANS_CHECKED, _err_ptr(err), _stream(),
    )


def host_stream_attention_table(q: torch.Tensor, out: torch.Tensor, table: np.ndarray,
                                num_kv_heads: int, q_start: int = 0, causal: bool = True,
                                scale: float | None = None, workspace: Workspace | None = None,
                                err: torch.Tensor | None = None) -> torch.Tensor:
    """host_stream_attention over a span table the caller has already built and checked.

    `table` is a uint64 [n, 6] array, one row per span in sequence order: K address, V
    address, length T, then the element strides of the [H_kv, T, D] views (head, token,
    dim). Every span must be device memory on q's GPU or page-locked host memory, in q's
    dtype with `num_kv_heads` heads and q's head_dim, and stay allocated until the launch
    has run; nothing here re-checks them. This is the per-step path of a decode loop that
    keeps its host chunks' rows across steps (decode.HostStoreDecoder): building the table
    is a few array operations instead of per-span tensor checks. q and out are
    [q_len, Hq, D] on the GPU with contiguous heads.
    """
    if q.dim() != 3 or out.shape != q.shape or out.dtype != q.dtype:
        raise ValueError("q and out must both be [q_len, Hq, D] in one dtype")
    if q.stride(2) != 1 or q.stride(1) != q.shape[2] or out.stride(2) != 1 \
            or out.stride(1) != q.shape[2]:
        raise ValueError("q and out need contiguous heads")
    _require_cuda(q, out)
    if table.dtype != np.uint64 or table.ndim != 2 or table.shape[1] != 6 or not table.flags.c_contiguous:
        raise ValueError("table must be a C-contiguous uint64 [n, 6] array")
    n = table.shape[0]
    if n > _capi.HS_MAX_SPANS:
        raise ValueError(f"at most {_capi.HS_MAX_SPANS} spans per call")
    if q.shape[1] % num_kv_heads:
        raise ValueError(f"Hq={q.shape[1]} is not a multiple of H_kv={num_kv_heads}")
    kv_len = int(table[:, 2].sum()) if n else 0
    if n == 0:
        table = np.array([(0, 0, 0, 0, 0, 1)], dtype=np.uint64)
    _host_stream_launch(q, out, table, n, num_kv_heads, kv_len, q_start, causal, scale,
                        workspace, err)
    return out


# ---------------------------------------------------------------------------
# e: decode attention with the all-gather fused in (multi-GPU, peer stores)
# ---------------------------------------------------------------------------


def paged_decode_attention_gather(
    q: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_tables: torch.Tensor,
    ctx_lens: torch.Tensor,
    exchange,
    scale: float | None = None,
    workspace: Workspace | None = None,
    err: torch.Tensor | None = None,
) -> torch.Tensor:
    """This rank's heads of decode attention, all-gathered across ranks in-kernel.

    `exchange` is a dist.PeerExchange built for (B, Hq_local, D). Returns the gathered
    [world * B, Hq_local, D] buffer (rank-major), complete (every rank's rows) for the
    work that follows on the current stream: the launch ends only after every rank's
    slice has landed (bounded wait; `err` gets PI_ERR_TIMEOUT if a rank never launches).
    """
    P, Hkv, S, D = _check_pool(k_pool, "k_pool")
    B, Hq, _ = q.shape
    if q.dtype != k_pool.dtype or q.shape[2] != D:
        raise ValueError("q must be [B, Hq_local, D] in the pool dtype")
    if exchange.shape != (exchange.world * B, Hq, D) or exchange.dtype != q.dtype:
        raise ValueError("exchange was built for another shape or dtype")
    _require_cuda(q, k_pool, v_pool, block_tables, ctx_lens)
    q = q.contiguous()
    block_tables = block_tables.contiguous()
    ctx_lens = ctx_lens.contiguous()
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    ex = exchange
    slot, g = ex.next_launch()
    gathered = ex.slot_tensor(slot)
    out = gathered[ex.rank * B:(ex.rank + 1) * B]
    nbytes = workspace_bytes(B, Hq, Hkv, D)
    ws = (workspace or default_workspace(q.device)).get(nbytes)
    _capi.call(
        "pi_paged_decode_attn_gather",
        out.data_ptr(), q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(),
        block_tables.data_ptr(), block_tables.stride(0), ctx_lens.data_ptr(),
        B, Hq, Hkv, D, S, P, float(scale), dtype_code(q.dtype), q.stride(0), out.stride(0),
        ws.data_ptr(), ws.numel(), ctypes.byref(g), _err_ptr(err), _stream(),
    )
    return gathered
