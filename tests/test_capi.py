"""The C-ABI library builds, loads, and exports exactly what include/plastic_kv.h declares.

No kernel is launched here (no GPU needed): only symbol presence, the ABI version,
status strings, and host-side argument validation, which returns before any CUDA
call.
"""

from __future__ import annotations

import ctypes
import pathlib
import re

import pytest

from plastic_infer_b200 import _build, _capi

HEADER = pathlib.Path(__file__).resolve().parent.parent / "include" / "plastic_kv.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pi_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib() -> ctypes.CDLL:
    _build.build()
    return _capi.load()


def test_header_and_binding_agree() -> None:
    assert declared_functions() == sorted(_capi.SIGNATURES)


def test_every_declared_symbol_is_exported(lib: ctypes.CDLL) -> None:
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_exports_are_the_declared_symbols(lib: ctypes.CDLL) -> None:
    # every exported pi_* symbol is declared in the header, and nothing else is exported
    import shutil
    import subprocess

    nm = shutil.which("nm")
    if nm is None:
        pytest.skip("nm not available")
    out = subprocess.run([nm, "-D", "--defined-only", str(_capi.lib_path())], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T pi_" in line}
    assert exported == set(declared_functions())


def test_version_and_strings(lib: ctypes.CDLL) -> None:
    assert lib.pi_abi_version() == _capi.ABI_VERSION
    for code in range(0, 10):
        s = _capi.error_string(code)
        assert s and s != "unknown status code"
    assert _capi.error_string(1234) == "unknown status code"


def test_host_validation_rejects_before_launch(lib: ctypes.CDLL) -> None:
    # zero tokens is a no-op
    assert lib.pi_kv_index_copy(None, None, None, None, None, 0, 8, 128, 16, 1024,
                                _capi.PI_DTYPE_BF16, 1024, None, None) == _capi.PI_OK
    # null pointers with work to do
    assert lib.pi_kv_index_copy(None, None, None, None, None, 4, 8, 128, 16, 1024,
                                _capi.PI_DTYPE_BF16, 1024, None, None) == _capi.PI_ERR_NULL_POINTER
    # unknown dtype
    assert lib.pi_kv_index_copy(None, None, None, None, None, 4, 8, 128, 16, 1024, 7, 1024,
                                None, None) == _capi.PI_ERR_UNSUPPORTED
    # token stride shorter than a row
    assert lib.pi_kv_index_copy(None, None, None, None, None, 4, 8, 128, 16, 1024,
                                _capi.PI_DTYPE_BF16, 100, None, None) == _capi.PI_ERR_BAD_SHAPE
    # Hq not a multiple of Hkv
    assert lib.pi_paged_decode_attn(None, None, None, None, None, 4, None, 2, 6, 4, 128, 16, 64,
                                    1.0, _capi.PI_DTYPE_BF16, 768, 768, None, 0, None,
                                    None) == _capi.PI_ERR_BAD_SHAPE
    # page moves: tile size not a multiple of 16 bytes
    fake = ctypes.c_void_p(256)
    assert lib.pi_page_gather(fake, fake, fake, 1, 2, 24, 1, 4, None,
                              None) == _capi.PI_ERR_MISALIGNED
    assert lib.pi_page_scatter(None, None, None, 0, 2, 4096, 1, 4, None, None) == _capi.PI_OK
    # fused decode prologue: head_dim 96 unsupported; nothing to do; null pointers
    pro = lib.pi_decode_prologue
    assert pro(fake, 1024, fake, fake, fake, 1024, fake, fake, 256, _capi.PI_DTYPE_BF16, None,
               None, 1e-5, fake, fake, fake, 4, 8, 2, 96, 16, 64, _capi.PI_DTYPE_BF16, None,
               None) == _capi.PI_ERR_UNSUPPORTED
    assert pro(None, 1024, None, None, None, 1024, None, None, 256, _capi.PI_DTYPE_BF16, None,
               None, 1e-5, None, None, None, 0, 8, 2, 128, 16, 64, _capi.PI_DTYPE_BF16, None,
               None) == _capi.PI_OK
    assert pro(None, 1024, None, None, None, 1024, None, None, 256, _capi.PI_DTYPE_BF16, None,
               None, 1e-5, None, None, None, 4, 8, 2, 128, 16, 64, _capi.PI_DTYPE_BF16, None,
               None) == _capi.PI_ERR_NULL_POINTER
    # one QK-norm weight without the other
    assert pro(fake, 1024, fake, fake, fake, 1024, fake, fake, 256, _capi.PI_DTYPE_BF16, fake,
               None, 1e-5, fake, fake, fake, 4, 8, 2, 128, 16, 64, _capi.PI_DTYPE_BF16, None,
               None) == _capi.PI_ERR_NULL_POINTER
    # request stride shorter than the q heads
    assert pro(fake, 1024, fake, fake, fake, 100, fake, fake, 256, _capi.PI_DTYPE_BF16, None,
               None, 1e-5, fake, fake, fake, 4, 8, 2, 128, 16, 64, _capi.PI_DTYPE_BF16, None,
               None) == _capi.PI_ERR_BAD_SHAPE
    # paged prefill: head_dim 256 and fp32 unsupported; group 3 unsupported; kv_len beyond
    # the block table; nothing to do
    pf = lib.pi_paged_prefill_attn
    args = lambda q_len, kv, hq, hkv, D, S, dt, tl: (  # noqa: E731
        fake, fake, fake, fake, fake, tl, q_len, kv, 0, 1, hq, hkv, D, S, 64, 1.0, dt, hq * D,
        hq * D, None, None)
    assert pf(*args(4, 16, 8, 2, 256, 16, _capi.PI_DTYPE_BF16, 1)) == _capi.PI_ERR_UNSUPPORTED
    assert pf(*args(4, 16, 8, 2, 128, 16, _capi.PI_DTYPE_F32, 1)) == _capi.PI_ERR_UNSUPPORTED
    assert pf(*args(4, 16, 6, 2, 128, 16, _capi.PI_DTYPE_BF16, 1)) == _capi.PI_ERR_UNSUPPORTED
    assert pf(*args(4, 17, 8, 2, 128, 16, _capi.PI_DTYPE_BF16, 1)) == _capi.PI_ERR_BAD_SHAPE
    assert pf(*args(0, 16, 8, 2, 128, 16, _capi.PI_DTYPE_BF16, 1)) == _capi.PI_OK
    # tcgen05 prefill: q and out move by TMA, so both need 16-byte aligned bases and token
    # strides that are multiples of 8 elements
    tc = lib.pi_paged_prefill_attn_tc
    assert tc(*args(0, 16, 8, 2, 128, 16, _capi.PI_DTYPE_BF16, 1)) == _capi.PI_OK
    ok = list(args(4, 16, 8, 2, 128, 16, _capi.PI_DTYPE_BF16, 1))
    for i, bad in ((0, ctypes.c_void_p(260)), (1, ctypes.c_void_p(264)), (17, 8 * 128 + 4),
                   (18, 8 * 128 + 2)):
        a = list(ok)
        a[i] = bad
        assert tc(*a) == _capi.PI_ERR_MISALIGNED, i
    # expert-slot copy: too many banks; nothing to do; null pointers
    ec = lib.pi_expert_slot_copy
    assert ec(fake, fake, fake, 33, fake, fake, 4, None, 1, None, None) == _capi.PI_ERR_BAD_SHAPE
    assert ec(None, None, None, 2, None, None, 0, None, 1, None, None) == _capi.PI_OK
    assert ec(None, fake, fake, 2, fake, fake, 4, None, 1, None, None) == _capi.PI_ERR_NULL_POINTER
    # arrival counters (4096 requests x 64 KV heads) + the grid-completion counter block
    assert lib.pi_paged_decode_attn_ws_zero_bytes() == 4096 * 64 * 4 + 256
    # host-stream attention: dtype, head_dim, head ratio, span count, nothing to do, nulls
    hs = lib.pi_host_stream_attn
    sp = (_capi.KvSpan * 1)(_capi.KvSpan(fake, fake, 4, 512, 64, 1))
    spp = ctypes.addressof(sp)
    hargs = lambda q_len, hq, hkv, D, dt, n=1, spans=spp, out=fake: (  # noqa: E731
        out, fake, hq * D, hq * D, spans, n, q_len, 0, 1, hq, hkv, D, 1.0, dt, None, 0, 0, None,
        None)
    assert hs(*hargs(1, 8, 2, 128, 7)) == _capi.PI_ERR_UNSUPPORTED
    assert hs(*hargs(1, 8, 2, 12, _capi.PI_DTYPE_BF16)) == _capi.PI_ERR_UNSUPPORTED
    assert hs(*hargs(1, 8, 2, 512, _capi.PI_DTYPE_BF16)) == _capi.PI_ERR_UNSUPPORTED
    assert hs(*hargs(1, 6, 4, 128, _capi.PI_DTYPE_BF16)) == _capi.PI_ERR_BAD_SHAPE
    assert hs(*hargs(1, 8, 2, 128, _capi.PI_DTYPE_BF16, n=_capi.HS_MAX_SPANS + 1)) == \
        _capi.PI_ERR_UNSUPPORTED
    assert hs(*hargs(0, 8, 2, 128, _capi.PI_DTYPE_F32)) == _capi.PI_OK
    assert hs(*hargs(1, 8, 2, 128, _capi.PI_DTYPE_F32, spans=None)) == _capi.PI_ERR_NULL_POINTER
    assert hs(*hargs(1, 8, 2, 128, _capi.PI_DTYPE_F32, out=None)) == _capi.PI_ERR_NULL_POINTER
    assert ctypes.sizeof(_capi.KvSpan) == 48


def test_kernels_refuse_cpu_tensors() -> None:
    import torch

    from plastic_infer_b200 import kernels

    pool = torch.zeros(4, 2, 16, 64, dtype=torch.bfloat16)
    new = torch.zeros(1, 2, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        kernels.kv_index_copy(pool, pool, new, new, torch.zeros(1, dtype=torch.int64))
    # host-stream attention: the query must be on the GPU (host chunks may not be)
    from plastic_infer_b200.exec.attention import host_stream_attention_v1

    q = torch.zeros(1, 1, 4, 64)
    chunk = (torch.zeros(2, 64, 8), torch.zeros(2, 64, 8))
    with pytest.raises(ValueError, match="CUDA"):
        kernels.host_stream_attention(q[0], [(chunk[0].permute(0, 2, 1), chunk[1].permute(0, 2, 1))])
    with pytest.raises(ValueError, match="CUDA"):
        host_stream_attention_v1(q, [chunk], torch.zeros(1, 0, 2, 64), torch.zeros(1, 0, 2, 64))
