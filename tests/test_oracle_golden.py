"""Pin the CPU oracle against golden vectors produced by the reference itself.

tests/golden/make_golden.py ran the reference's own functions (append_token,
_write_kv_layer, paged_attention_v1, sink_completed_chunks, load_prefix,
compute_prefix_hashes, qk_norm + rope_positions, _attn_paged prefill) on seeded inputs;
here the numpy
restatement must reproduce every one of those results (bit-exact for copies, 1e-5 for
fp32 attention and the fp32 decode prologue).
"""

from __future__ import annotations

import json
import pathlib

import numpy as np
import pytest

from oracle import paged_kv_oracle as orc
from tests.golden.inputs import (
    ATTENTION_CASES, HOST_STREAM_CASES, PREFILL_CASES, PROLOGUE_CASES, attention_inputs, checksum,
    host_stream_inputs, prefill_inputs, prologue_inputs,
)

GOLD = pathlib.Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_index_copy_matches_reference(dtype: str) -> None:
    g = np.load(GOLD / f"index_copy_{dtype}.npz")
    k = np.zeros_like(g["k_pages"])
    v = np.zeros_like(g["v_pages"])
    orc.write_kv_slots(k, v, g["k_new"], g["v_new"], g["slots"], int(g["page_size"]))
    assert np.array_equal(k, g["k_pages"])
    assert np.array_equal(v, g["v_pages"])


@pytest.mark.parametrize("case", ATTENTION_CASES, ids=[c["name"] for c in ATTENTION_CASES])
def test_attention_matches_reference(case: dict) -> None:
    g = np.load(GOLD / "attention.npz")
    x = attention_inputs(case)
    assert checksum(x["q"], x["k"], x["v"]) == pytest.approx(float(g[case["name"] + "/checksum"]),
                                                            rel=1e-12)
    out = orc.paged_attention_decode(x["q"], x["k"], x["v"], x["tables"], x["ctx"], case["S"])
    ref = g[case["name"] + "/out"]
    np.testing.assert_allclose(out, ref, atol=2e-5, rtol=1e-5)


@pytest.mark.parametrize("case", ATTENTION_CASES, ids=[c["name"] for c in ATTENTION_CASES])
def test_reference_torch_path_matches_reference(case: dict) -> None:
    # The timed reference arm (the reference's torch operations, restated) reproduces the
    # reference's own attention outputs on the same fp32 inputs.
    import torch

    from oracle import ref_torch_path as rtp

    g = np.load(GOLD / "attention.npz")
    x = attention_inputs(case)
    kp, vp = torch.from_numpy(x["k"]), torch.from_numpy(x["v"])
    q = torch.from_numpy(x["q"])
    out = np.stack([
        rtp.decode_attention(q[b].view(1, 1, *q.shape[1:]), kp, vp,
                             x["tables"][b][:-(-n // case["S"])], case["S"], n)[0, 0].numpy()
        for b, n in enumerate(x["ctx"])])
    np.testing.assert_allclose(out, g[case["name"] + "/out"], atol=2e-5, rtol=1e-5)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_reference_torch_path_write_matches_reference(dtype: str) -> None:
    import torch

    from oracle import ref_torch_path as rtp

    g = np.load(GOLD / f"index_copy_{dtype}.npz")
    S = int(g["page_size"])
    conv = ((lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16))
            if dtype == "bf16" else torch.from_numpy)
    k = torch.zeros_like(conv(g["k_pages"]))
    v = torch.zeros_like(k)
    kn, vn = conv(g["k_new"]), conv(g["v_new"])
    for i, s in enumerate(g["slots"].tolist()):
        rtp.write_kv_token(k, v, s // S, s % S, kn[i], vn[i])
    back = (lambda t: t.view(torch.int16).numpy().view(np.uint16)) if dtype == "bf16" else (
        lambda t: t.numpy())
    assert np.array_equal(back(k), g["k_pages"])
    assert np.array_equal(back(v), g["v_pages"])


def test_reference_torch_path_decode_layer_matches_oracle() -> None:
    # write-then-attend over a batch: the reference arm's step equals the oracle's
    import torch

    from oracle import ref_torch_path as rtp

    rng = np.random.default_rng(4)
    B, Hq, Hkv, D, S = 5, 8, 2, 64, 16
    ctx = [1, 16, 17, 40, 0]
    npg = [-(-n // S) for n in ctx]
    P = sum(npg) + 2
    perm = rng.permutation(P)
    tables, cur = [], 0
    for n in npg:
        tables.append([int(x) for x in perm[cur:cur + n]])
        cur += n
    kp = rng.standard_normal((P, Hkv, D, S), dtype=np.float32)
    vp = rng.standard_normal((P, Hkv, D, S), dtype=np.float32)
    q = rng.standard_normal((B, Hq, D), dtype=np.float32)
    kn = rng.standard_normal((B, Hkv, D), dtype=np.float32)
    vn = rng.standard_normal((B, Hkv, D), dtype=np.float32)
    tk, tv = torch.from_numpy(kp.copy()), torch.from_numpy(vp.copy())
    got = rtp.decode_layer(torch.from_numpy(q), torch.from_numpy(kn), torch.from_numpy(vn), tk, tv,
                           tables, ctx, S).numpy()
    slots = np.array([orc.slot_of(t, n - 1, S) if n > 0 else -1 for t, n in zip(tables, ctx)])
    orc.write_kv_slots(kp, vp, kn, vn, slots, S)
    ref = orc.paged_attention_decode(q, kp, vp, tables, ctx, S)
    assert np.array_equal(tk.numpy(), kp)
    np.testing.assert_allclose(got, ref, atol=2e-5, rtol=1e-5)


def test_gather_matches_reference_layout() -> None:
    # gather_paged_kv of a non-contiguous table [4, 1, 3] with a partial last page
    # (tests/test_ops.py:227-266 geometry) == page-by-page permute + concat.
    rng = np.random.default_rng(0)
    kp = rng.standard_normal((5, 2, 8, 3)).astype(np.float32)
    vp = rng.standard_normal((5, 2, 8, 3)).astype(np.float32)
    k, v = orc.gather_paged_kv(kp, vp, [4, 1, 3], 3, num_tokens=8)
    ref = np.concatenate([kp[p].transpose(2, 0, 1) for p in [4, 1, 3]])[:8]
    assert np.array_equal(k, ref)
    e, _ = orc.gather_paged_kv(kp, vp, [], 3)
    assert e.shape == (0, 2, 8)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_sink_and_load_match_reference(dtype: str) -> None:
    g = np.load(GOLD / f"store_{dtype}.npz")
    L, H, D, S, ppc, P = (int(g[k]) for k in ("L", "H", "D", "S", "ppc", "P"))
    from tests.golden.inputs import token_kv
    from oracle.paged_kv_oracle import f32_to_bf16_bits

    ntok = len(g["tokens"])
    k, v = token_kv(21 if dtype == "f32" else 22, ntok, L, H, D, dtype)
    if dtype == "bf16":
        k, v = f32_to_bf16_bits(k), f32_to_bf16_bits(v)
    # Replay the appends into a logical pool with the recorded tables.
    pool_dt = np.uint16 if dtype == "bf16" else np.float32
    kp = np.zeros((P, H, D, S), pool_dt)
    vp = np.zeros((P, H, D, S), pool_dt)
    tables = [list(map(int, r)) for r in g["c1_tables"]]
    for layer in range(L):
        slots = [orc.slot_of(tables[layer], t, S) for t in range(ntok)]
        orc.write_kv_slots(kp, vp, k[:, layer], v[:, layer], np.asarray(slots), S)
    n_chunks = int(g["sunk"])
    for c in range(n_chunks):
        kc, vc = orc.sink_chunk(kp, vp, tables, c, S, ppc)
        assert np.array_equal(kc, g["host_k"][c])
        assert np.array_equal(vc, g["host_v"][c])
    # Load into the recorded fresh pages and compare the pool contents.
    kp2 = np.zeros_like(kp)
    vp2 = np.zeros_like(vp)
    c2 = [list(map(int, r)) for r in g["c2_tables"]]
    for c in range(int(g["matched"]) // (S * ppc)):
        orc.load_chunk(kp2, vp2, g["host_k"][c], g["host_v"][c],
                       [row[c * ppc:(c + 1) * ppc] for row in c2], S)
    for layer in range(L):
        assert np.array_equal(kp2[c2[layer]], g["loaded_k"][layer])
        assert np.array_equal(vp2[c2[layer]], g["loaded_v"][layer])


def test_chunk_keys_match_reference() -> None:
    gold = json.loads((GOLD / "chunk_keys.json").read_text())
    for name, case in gold.items():
        keys = orc.chunk_keys(case["tokens"], case["chunk_size"])
        assert [p.hex() for p, _ in keys] == case["prefix"], name
        assert [c.hex() for _, c in keys] == case["cumulative"], name


def test_bf16_rounding_is_round_to_nearest_even() -> None:
    import torch

    x = np.random.default_rng(1).standard_normal(4096).astype(np.float32) * 100
    x[:4] = [1.00390625, 1.01171875, -2.0078125, 3.0e38]  # exact ties and a large value
    bits = orc.f32_to_bf16_bits(x)
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(bits, ref)


@pytest.mark.parametrize("case", PROLOGUE_CASES, ids=[c["name"] for c in PROLOGUE_CASES])
def test_decode_prologue_matches_reference(case: dict) -> None:
    g = np.load(GOLD / "prologue.npz")
    n = case["name"]
    x = prologue_inputs(case)
    assert checksum(*(x[k] for k in sorted(x))) == pytest.approx(float(g[n + "__checksum"]), rel=1e-12)
    q, k, v = orc.decode_prologue(x["q"], x["k"], x["v"], x["positions"], g[n + "__inv_freq"],
                                  x.get("q_norm_w"), x.get("k_norm_w"))
    # fp32 both sides; cos/sin of angles up to ~3e4 rad differ by an ulp between libms
    np.testing.assert_allclose(q, g[n + "__q"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(k, g[n + "__k"], rtol=1e-5, atol=1e-5)
    assert np.array_equal(v, x["v"])


@pytest.mark.parametrize("case", PROLOGUE_CASES, ids=[c["name"] for c in PROLOGUE_CASES])
def test_rope_inv_freq_is_the_reference_table_frequency(case: dict) -> None:
    # the product path's frequencies are bit-identical to the reference's fp32 table's
    from plastic_infer_b200.kernels import rope_inv_freq

    g = np.load(GOLD / "prologue.npz")
    assert np.array_equal(rope_inv_freq(case["D"], case["base"]).numpy(),
                          g[case["name"] + "__inv_freq"])


def prefill_pools(case: dict, x: dict, table: np.ndarray):
    """Logical [P, H, D, S] pools holding the context's K/V rows at the table's pages."""
    S, Hkv, D = case["S"], case["Hkv"], case["D"]
    P = int(table.max()) + 1 if len(table) else 1
    k = np.zeros((P, Hkv, D, S), dtype=np.float32)
    v = np.zeros_like(k)
    for t in range(case["kv_len"]):
        k[table[t // S], :, :, t % S] = x["k"][t]
        v[table[t // S], :, :, t % S] = x["v"][t]
    return k, v


@pytest.mark.parametrize("case", PREFILL_CASES, ids=[c["name"] for c in PREFILL_CASES])
def test_prefill_matches_reference(case: dict) -> None:
    g = np.load(GOLD / "prefill.npz")
    n = case["name"]
    x = prefill_inputs(case)
    assert checksum(x["q"], x["k"], x["v"]) == pytest.approx(float(g[n + "__checksum"]), rel=1e-12)
    table = g[n + "__table"]
    k, v = prefill_pools(case, x, table)
    out = orc.paged_attention_prefill(x["q"], k, v, list(table), case["kv_len"], case["q_start"],
                                      case["causal"], case["S"])
    np.testing.assert_allclose(out, g[n + "__out"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("case", HOST_STREAM_CASES, ids=[c["name"] for c in HOST_STREAM_CASES])
def test_host_stream_matches_reference(case: dict) -> None:
    # host_stream_attention_v1 run by the reference on the same chunks (CPU fp32)
    g = np.load(GOLD / "host_stream.npz")
    n = case["name"]
    x = host_stream_inputs(case)
    assert checksum(x["q"], x["k_full"], x["v_full"]) == pytest.approx(
        float(g[n + "__checksum"]), rel=1e-12)
    out = orc.host_stream_attention(x["q"], x["chunks"], x["rk"], x["rv"], case["q_start"],
                                    case["causal"])
    np.testing.assert_allclose(out, g[n + "__out"], rtol=1e-5, atol=1e-6)


def test_host_stream_oracle_is_contiguous_attention() -> None:
    # the chunk split is invisible: one contiguous span gives the same rows
    case = HOST_STREAM_CASES[4]
    x = host_stream_inputs(case)
    whole = orc.host_stream_attention(x["q"], [], x["k_full"], x["v_full"], case["q_start"],
                                      case["causal"])
    split = orc.host_stream_attention(x["q"], x["chunks"], x["rk"], x["rv"], case["q_start"],
                                      case["causal"])
    np.testing.assert_allclose(split, whole, rtol=1e-6, atol=1e-7)
