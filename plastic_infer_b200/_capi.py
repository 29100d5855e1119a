"""ctypes binding of libplastic_kv.so (declared in include/plastic_kv.h).

Mirrors the reference's ctypes binding idiom (src/plastic_infer/kernel/jit.py:87-124,
src/plastic_infer/kernel/fast_index_copy.py:88-186): plain pointers, sizes and the
caller's CUDA stream handle. Unlike the reference, every entry point returns a
status that is turned into an exception here.

There is no fallback: if the library is missing or cannot be loaded, every kernel
call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

from . import _build

PI_OK = 0
PI_ERR_NULL_POINTER = 1
PI_ERR_BAD_SHAPE = 2
PI_ERR_MISALIGNED = 3
PI_ERR_UNSUPPORTED = 4
PI_ERR_CUDA = 5
PI_ERR_WORKSPACE = 6
PI_ERR_SLOT_RANGE = 7
PI_ERR_PAGE_RANGE = 8
PI_ERR_TIMEOUT = 9
PI_ERR_SCRATCH_LIMIT = 10
NOALLOC_SCRATCH_BYTES = 12 << 20  # PI_NOALLOC_SCRATCH_BYTES in include/plastic_kv.h

PI_ATTN_RING_AUTO = 0
PI_ATTN_RING_DEEP = 1
PI_ATTN_RING_SHALLOW = 2

PI_DTYPE_F32 = 0
PI_DTYPE_BF16 = 1
PI_DTYPE_F16 = 2

ABI_VERSION = 3

_vp = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t
_f32 = ctypes.c_float

# name -> (restype, argtypes); the one table of what the header declares.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "pi_set_programmatic_launch": (_i32, [_i32]),
    "pi_set_decode_attn_ring": (_i32, [_i32]),
    "pi_abi_version": (_i32, []),
    "pi_error_string": (ctypes.c_char_p, [_i32]),
    "pi_kv_index_copy": (
        _i32,
        [_vp, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i64, _i32, _i64, _vp, _vp],
    ),
    "pi_paged_decode_attn_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32]),
    "pi_paged_decode_attn_ws_zero_bytes": (_sz, []),
    # batch, bt_stride, hq, hkv, head_dim, page_size, num_pages, dtype
    "pi_paged_decode_attn_ring_stages": (_i32, [_i32, _i64, _i32, _i32, _i32, _i32, _i64, _i32]),
    "pi_paged_decode_attn": (
        _i32,
        [_vp, _vp, _vp, _vp, _vp, _i64, _vp, _i32, _i32, _i32, _i32, _i32, _i64, _f32, _i32,
         _i64, _i64, _vp, _sz, _vp, _vp],
    ),
    "pi_paged_decode_attn_gather": (
        _i32,
        [_vp, _vp, _vp, _vp, _vp, _i64, _vp, _i32, _i32, _i32, _i32, _i32, _i64, _f32, _i32,
         _i64, _i64, _vp, _sz, _vp, _vp, _vp],
    ),
    "pi_paged_decode_attn_append": (
        _i32,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _vp, _i32, _i32, _i32, _i32, _i32,
         _i64, _f32, _i32, _i64, _i64, _vp, _sz, _vp, _vp],
    ),
    # allocation-free variant: scratch is the library's built-in array (no workspace)
    "pi_paged_decode_attn_noalloc": (
        _i32,
        [_vp, _vp, _vp, _vp, _vp, _i64, _vp, _i32, _i32, _i32, _i32, _i32, _i64, _f32, _i32,
         _i64, _i64, _vp, _vp],
    ),
    # out, q, k_pool, v_pool, block_table, table_len, q_len, kv_len, q_start, causal, hq,
    # hkv, head_dim, page_size, num_pages, scale, dtype, q_tok_stride, out_tok_stride, err,
    # stream
    "pi_paged_prefill_attn": (
        _i32,
        [_vp, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i64,
         _f32, _i32, _i64, _i64, _vp, _vp],
    ),
    # same arguments as pi_paged_prefill_attn (tcgen05 kernel)
    "pi_paged_prefill_attn_tc": (
        _i32,
        [_vp, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i64,
         _f32, _i32, _i64, _i64, _vp, _vp],
    ),
    # dst_ptrs, src_ptrs, feat_bytes, num_banks, dst_indices, src_indices, length,
    # num_indices, use_int32, err, stream
    "pi_expert_slot_copy": (_i32, [_vp, _vp, _vp, _i32, _vp, _vp, _i64, _vp, _i32, _vp, _vp]),
    # q_out, q_out_stride, k_pool, v_pool, q_in, q_in_stride, k_in, v_in, kv_in_stride,
    # in_dtype, q_norm_w, k_norm_w, eps, inv_freq, positions, slot_mapping, batch, hq, hkv,
    # head_dim, page_size, num_slots, pool_dtype, err, stream
    "pi_decode_prologue": (
        _i32,
        [_vp, _i64, _vp, _vp, _vp, _i64, _vp, _vp, _i64, _i32, _vp, _vp, _f32, _vp, _vp, _vp,
         _i32, _i32, _i32, _i32, _i32, _i64, _i32, _vp, _vp],
    ),
    # q_len, num_q_heads, num_kv_heads, head_dim, kv_len
    "pi_host_stream_attn_workspace_size": (_sz, [_i32, _i32, _i32, _i32, _i64]),
    # out, q, q_tok_stride, out_tok_stride, spans (host array), num_spans, q_len, q_start,
    # causal, hq, hkv, head_dim, scale, dtype, workspace, workspace_bytes, flags, err, stream
    "pi_host_stream_attn": (
        _i32,
        [_vp, _vp, _i64, _i64, _vp, _i32, _i32, _i64, _i32, _i32, _i32, _i32, _f32, _i32, _vp,
         _sz, _i32, _vp, _vp],
    ),
    "pi_paged_kv_gather": (_i32, [_vp, _vp, _vp, _i64, _i32, _i32, _i32, _i64, _i32, _vp, _vp]),
    "pi_page_gather": (_i32, [_vp, _vp, _vp, _i64, _i32, _i64, _i32, _i64, _vp, _vp]),
    "pi_page_scatter": (_i32, [_vp, _vp, _vp, _i64, _i32, _i64, _i32, _i64, _vp, _vp]),
}

MAX_PEERS = 8  # PI_MAX_PEERS


class PeerGather(ctypes.Structure):
    """pi_peer_gather_t (include/plastic_kv.h)."""

    _fields_ = [
        ("peer_out", ctypes.c_void_p * MAX_PEERS),
        ("peer_flags", ctypes.c_void_p * MAX_PEERS),
        ("rank", ctypes.c_int),
        ("world", ctypes.c_int),
        ("rank_stride", ctypes.c_int64),
        ("epoch", ctypes.c_uint),
        ("launch_counter", ctypes.c_void_p),
    ]


HS_MAX_SPANS = 512  # PI_HS_MAX_SPANS
HS_SPANS_CHECKED = 1  # PI_HS_SPANS_CHECKED


class KvSpan(ctypes.Structure):
    """pi_kv_span_t (include/plastic_kv.h)."""

    _fields_ = [
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("len", ctypes.c_int64),
        ("head_stride", ctypes.c_int64),
        ("tok_stride", ctypes.c_int64),
        ("dim_stride", ctypes.c_int64),
    ]


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class KernelError(RuntimeError):
    """A libplastic_kv entry point returned a non-zero status."""

    def __init__(self, func: str, code: int, msg: str) -> None:
        super().__init__(f"{func} failed with status {code}: {msg}")
        self.code = code
        self.func = func


def lib_path() -> str:
    """The in-tree library, or the file named by PLASTIC_KV_LIB (e.g. a build with
    other compile-time tunables)."""
    return os.environ.get("PLASTIC_KV_LIB") or str(_build.LIB_PATH)


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raise if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not os.path.exists(path):
            raise RuntimeError(
                f"{path} is not built; run `python -m plastic_infer_b200._build` "
                "(the paged-KV path has no CPU or PyTorch fallback)"
            )
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        ver = lib.pi_abi_version()
        if ver != ABI_VERSION:
            raise RuntimeError(f"libplastic_kv ABI {ver} != expected {ABI_VERSION}; rebuild")
        _lib = lib
        return lib


def error_string(code: int) -> str:
    return load().pi_error_string(code).decode()


def check(func: str, code: int) -> None:
    if code != PI_OK:
        raise KernelError(func, code, error_string(code))


def call(func: str, *args) -> None:
    """Call a status-returning entry point and raise on failure."""
    check(func, getattr(load(), func)(*args))
