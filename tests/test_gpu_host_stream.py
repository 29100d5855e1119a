"""GPU parity of host-stream attention (pi_host_stream_attn).

One request attends over host chunks read in place (page-locked) plus a device tail,
in one pass: the reference's host_stream_attention_v1 (src/plastic_infer/exec/
attention.py:193-250) without its concatenation. Tolerances: fp32 runs against the
reference's own outputs (golden host_stream.npz) within 1e-4; bf16/f16 runs against
the oracle evaluated on exactly the values the kernel reads, within the attention bar
|err| <= 2e-2 + 1e-2 |ref|. Covered:
- the reference's cases with chunks pageable (copied to the GPU), pinned (read in
  place) and on the device;
- model shapes (G = 4 / 8, head_dim 128) in bf16 and f16, decode and offset suffixes;
- a 40k-token sequence in 157 spans (many splits and their merge);
- host chunks in the reference's [H_kv, D, C] layout next to token-major ones;
- no keys at all, a strided q and an out= buffer, pageable spans refused;
- the KV store end to end: sink, evict (the fixed eviction: a later request reuses the
  freed pages), then attend the evicted request from its host copies.
"""

from __future__ import annotations

import ctypes
import pathlib

import numpy as np
import pytest
import torch

from oracle import paged_kv_oracle as orc
from plastic_infer_b200 import _capi, kernels
from plastic_infer_b200.exec.attention import host_stream_attention_v1
from plastic_infer_b200.kv.kv_store import KVConfig, KVStore
from tests.golden.inputs import HOST_STREAM_CASES, host_stream_inputs

pytestmark = pytest.mark.gpu
GOLD = pathlib.Path(__file__).resolve().parent / "golden"
DEV = torch.device("cuda", 0)
ATOL, RTOL = 2e-2, 1e-2


def _close(got: np.ndarray, ref: np.ndarray, atol: float = ATOL, rtol: float = RTOL) -> None:
    err = np.abs(got - ref)
    bad = err > atol + rtol * np.abs(ref)
    assert not bad.any(), f"max abs err {err.max():.3e}, {int(bad.sum())} of {bad.size} outside"


@pytest.mark.parametrize("place", ["pageable", "pinned", "device"])
@pytest.mark.parametrize("case", HOST_STREAM_CASES, ids=[c["name"] for c in HOST_STREAM_CASES])
def test_matches_reference_golden(case: dict, place: str) -> None:
    g = np.load(GOLD / "host_stream.npz")
    x = host_stream_inputs(case)

    def put(a: np.ndarray) -> torch.Tensor:
        t = torch.from_numpy(a)
        return t.pin_memory() if place == "pinned" else (t.to(DEV) if place == "device" else t)

    chunks = [(put(kc), put(vc)) for kc, vc in x["chunks"]]
    q = torch.from_numpy(x["q"]).to(DEV)
    out = host_stream_attention_v1(q, chunks, torch.from_numpy(x["rk"]).to(DEV),
                                   torch.from_numpy(x["rv"]).to(DEV), q_start_pos=case["q_start"],
                                   causal=case["causal"])
    torch.cuda.synchronize()
    assert out.shape == (1, case["q_len"], case["Hq"], case["D"])
    _close(out.cpu().numpy(), g[case["name"] + "__out"], atol=1e-4, rtol=1e-4)


def _spans_token_major(k: np.ndarray, v: np.ndarray, cuts: list[int], dtype: torch.dtype,
                       tail_on_device: bool = True):
    """Cut a [kv, H, D] sequence into pinned host spans [H, T, D] (token-major, like the
    KV store's chunk buffers) at `cuts`, the last piece on the device."""
    kt = torch.from_numpy(k).to(dtype)
    vt = torch.from_numpy(v).to(dtype)
    spans = []
    edges = [0] + cuts + [k.shape[0]]
    for i, (a, b) in enumerate(zip(edges[:-1], edges[1:])):
        ks = kt[a:b].permute(1, 0, 2).contiguous()
        vs = vt[a:b].permute(1, 0, 2).contiguous()
        last = i == len(edges) - 2
        if last and tail_on_device:
            spans.append((ks.to(DEV), vs.to(DEV)))
        else:
            spans.append((ks.pin_memory(), vs.pin_memory()))
    # what the kernel reads, back in float32
    return spans, kt.float().numpy(), vt.float().numpy()


def _oracle(q: torch.Tensor, k: np.ndarray, v: np.ndarray, q_start: int, causal: bool) -> np.ndarray:
    qn = q.float().cpu().numpy()[None]
    return orc.host_stream_attention(qn, [], k[None], v[None], q_start, causal)[0]


CASES = [
    # (kv_len, cuts, q_len, q_start, causal, Hq, Hkv, D, dtype)
    (3000, [1024, 2048, 2944], 1, 3000, True, 32, 8, 128, torch.bfloat16),    # 8B decode
    (1500, [512, 1024], 7, 1400, True, 32, 4, 128, torch.bfloat16),           # MoE suffix
    (777, [256, 700], 1, 777, True, 64, 8, 128, torch.float16),               # G = 8, f16
    (333, [128], 5, 0, False, 16, 16, 64, torch.bfloat16),                    # MHA, non-causal
    (64, [32], 64, 0, True, 8, 2, 128, torch.bfloat16),                       # all rows causal
]


@pytest.mark.parametrize("kv,cuts,q_len,q_start,causal,Hq,Hkv,D,dtype", CASES)
def test_model_shapes_vs_oracle(kv, cuts, q_len, q_start, causal, Hq, Hkv, D, dtype) -> None:
    rng = np.random.default_rng(kv + q_len)
    k = rng.standard_normal((kv, Hkv, D), dtype=np.float32)
    v = rng.standard_normal((kv, Hkv, D), dtype=np.float32)
    spans, kf, vf = _spans_token_major(k, v, cuts, dtype)
    q = torch.from_numpy(rng.standard_normal((q_len, Hq, D), dtype=np.float32)).to(dtype).to(DEV)
    out = kernels.host_stream_attention(q, spans, q_start=q_start, causal=causal)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    _close(got, _oracle(q, kf, vf, q_start, causal))


@pytest.mark.parametrize("q_len", [1, 3])
def test_long_sequence_many_spans(q_len: int) -> None:
    kv, Hq, Hkv, D = 40000, 32, 8, 128
    rng = np.random.default_rng(40 + q_len)
    k = rng.standard_normal((kv, Hkv, D), dtype=np.float32)
    v = rng.standard_normal((kv, Hkv, D), dtype=np.float32)
    cuts = list(range(256, kv - 63, 256))           # 156 host chunks + a 64-token tail
    spans, kf, vf = _spans_token_major(k, v, cuts, torch.bfloat16)
    assert len(spans) == 157
    q = torch.from_numpy(rng.standard_normal((q_len, Hq, D), dtype=np.float32)).to(
        torch.bfloat16).to(DEV)
    q_start = kv - q_len
    out = kernels.host_stream_attention(q, spans, q_start=q_start, causal=True)
    torch.cuda.synchronize()
    _close(out.float().cpu().numpy(), _oracle(q, kf, vf, q_start, True))


def test_reference_layout_chunks_next_to_token_major() -> None:
    kv, Hq, Hkv, D = 200, 16, 4, 64
    rng = np.random.default_rng(5)
    k = rng.standard_normal((kv, Hkv, D), dtype=np.float32)
    v = rng.standard_normal((kv, Hkv, D), dtype=np.float32)
    kt = torch.from_numpy(k).half()
    vt = torch.from_numpy(v).half()
    # [0, 80): reference layout [H, D, C] pinned (strided element reads); [80, 150):
    # token-major pinned; [150, 200): device tail [1, R, H, D]
    ref_k = kt[:80].permute(1, 2, 0).contiguous().pin_memory()
    ref_v = vt[:80].permute(1, 2, 0).contiguous().pin_memory()
    tm_k = kt[80:150].permute(1, 0, 2).contiguous().pin_memory()
    tm_v = vt[80:150].permute(1, 0, 2).contiguous().pin_memory()
    spans = [(ref_k.permute(0, 2, 1), ref_v.permute(0, 2, 1)), (tm_k, tm_v),
             (kt[150:].permute(1, 0, 2).to(DEV), vt[150:].permute(1, 0, 2).to(DEV))]
    q = torch.from_numpy(rng.standard_normal((2, Hq, D), dtype=np.float32)).half().to(DEV)
    out = kernels.host_stream_attention(q, spans, causal=False)
    # and the reference API with the same chunks (layout [H, D, C]) and tail
    out_v1 = host_stream_attention_v1(q[None], [(ref_k, ref_v), (tm_k.permute(0, 2, 1),
                                                                 tm_v.permute(0, 2, 1))],
                                      kt[None, 150:].to(DEV), vt[None, 150:].to(DEV),
                                      q_start_pos=0, causal=False)
    torch.cuda.synchronize()
    ref = _oracle(q, kt.float().numpy(), vt.float().numpy(), 0, False)
    _close(out.float().cpu().numpy(), ref)
    assert torch.equal(out_v1[0], out)


def test_no_keys_strided_q_out_and_refusals() -> None:
    Hq, Hkv, D = 8, 2, 64
    q = torch.randn(3, Hq, D, dtype=torch.bfloat16, device=DEV)
    z = kernels.host_stream_attention(q, [], num_kv_heads=Hkv)
    empty = torch.empty(Hkv, 0, D, dtype=torch.bfloat16, device=DEV)
    z2 = kernels.host_stream_attention(q, [(empty, empty)])
    torch.cuda.synchronize()
    assert int(torch.count_nonzero(z)) == 0 and int(torch.count_nonzero(z2)) == 0
    # strided q (a fused-QKV slice) and a caller-provided out
    k = torch.randn(Hkv, 50, D, dtype=torch.bfloat16)
    vv = torch.randn(Hkv, 50, D, dtype=torch.bfloat16)
    spans = [(k.pin_memory(), vv.pin_memory())]
    qkv = torch.zeros(3, (Hq + 2 * Hkv) * D, dtype=torch.bfloat16, device=DEV)
    qkv[:, :Hq * D] = q.reshape(3, -1)
    out = torch.full((3, Hq, D), 5.0, dtype=torch.bfloat16, device=DEV)
    kernels.host_stream_attention(qkv[:, :Hq * D].view(3, Hq, D), spans, q_start=48, out=out)
    ref = kernels.host_stream_attention(q, spans, q_start=48)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    # pageable host memory has no device alias: refused by the wrapper and by the ABI
    with pytest.raises(ValueError, match="page-locked"):
        kernels.host_stream_attention(q, [(k, vv)])
    sp = (_capi.KvSpan * 1)(_capi.KvSpan(k.data_ptr(), vv.data_ptr(), 50, 50 * D, D, 1))
    rc = _capi.load().pi_host_stream_attn(
        out.data_ptr(), q.data_ptr(), Hq * D, Hq * D, ctypes.addressof(sp), 1, 3, 0, 1, Hq, Hkv, D,
        1.0, _capi.PI_DTYPE_BF16, None, 0, 0, None, None)
    assert rc == _capi.PI_ERR_UNSUPPORTED
    with pytest.raises(ValueError, match="at most"):
        kernels.host_stream_attention(q, spans * (_capi.HS_MAX_SPANS + 1))


def test_kv_store_evict_then_stream_from_host() -> None:
    # sink -> evict (fixed: no stale block-table entries) -> attend from the host copies
    L, H, D, S, ppc = 2, 2, 64, 16, 2
    store = KVStore(KVConfig(n_layers=L, n_kv_heads=H, head_dim=D, page_size=S,
                             pages_per_chunk=ppc, max_pages=64, dtype=torch.bfloat16, device=DEV))
    cache = store.new_request()
    n_tok = 5 * S * ppc + 10                              # 5 complete chunks + 10 tokens
    rng = np.random.default_rng(9)
    kk = rng.standard_normal((n_tok, L, H, D), dtype=np.float32)
    vv = rng.standard_normal((n_tok, L, H, D), dtype=np.float32)
    for t in range(n_tok):
        cache.append_token(torch.from_numpy(kk[t]).to(DEV), torch.from_numpy(vv[t]).to(DEV))
    cache.set_token_ids(list(range(n_tok)))
    assert store.sink_completed_chunks(cache) == 5
    evicted = {p for layer in range(L) for p in cache.get_block_table_for_layer(layer)[:2 * ppc]}
    freed = store.evict_chunks(need_pages=2 * L * ppc, protected_request=cache)
    assert freed == 2 * L * ppc and cache.evicted_chunks == 2
    # another request takes the freed pages and writes over them
    other = store.new_request()
    for t in range(2 * S * ppc):
        other.append_token(torch.full((L, H, D), 9.0, device=DEV),
                           torch.full((L, H, D), -9.0, device=DEV))
    reused = {p for layer in range(L) for p in other.get_block_table_for_layer(layer)}
    assert reused & evicted  # the stale-entry bug would now read the other request's rows
    assert all(p == -1 for p in cache.get_block_table_for_layer(0)[:2 * ppc])
    kb = torch.from_numpy(kk).to(torch.bfloat16).float().numpy()
    vb = torch.from_numpy(vv).to(torch.bfloat16).float().numpy()
    for layer in range(L):
        chunks, rk, rv = store.host_stream_chunks(cache, layer)
        assert len(chunks) == 2 and all(c.is_pinned() for c, _ in chunks)
        assert rk.shape == (1, n_tok - 2 * S * ppc, H, D)
        q = torch.randn(1, 1, 4 * H, D, dtype=torch.bfloat16, device=DEV)
        out = host_stream_attention_v1(q, chunks, rk, rv, q_start_pos=n_tok - 1)
        torch.cuda.synchronize()
        ref = _oracle(q[0], kb[:, layer], vb[:, layer], n_tok - 1, True)
        _close(out[0].float().cpu().numpy(), ref)
    store.free_request(cache)
    store.free_request(other)
    assert store.gpu.allocator.used_pages == 0
