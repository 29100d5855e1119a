"""Deterministic synthetic inputs shared by the golden-vector generator and the tests.

Golden files (tests/golden/*.npz) hold the reference's *outputs*; large inputs are
regenerated here from their seed with numpy's PCG64 (stable across machines) and
their checksum is stored beside the outputs so a generator change is caught.

bf16 tensors are carried as uint16 bit patterns (see oracle.paged_kv_oracle).
"""

from __future__ import annotations

import numpy as np

from oracle.paged_kv_oracle import bf16_bits_to_f32, f32_to_bf16_bits

# Attention parity cases: (name, seed, B, Hq, Hkv, D, S, num_pages, ctx_lens, dtype)
ATTENTION_CASES = [
    # C1 tiny shape (fp32): 4 ragged requests
    dict(name="att_c1_f32", seed=101, B=4, Hq=4, Hkv=2, D=64, S=16, P=24,
         ctx=[8, 23, 48, 64], dtype="f32"),
    # Qwen3-8B head shape (bf16): single token, partial page, several pages
    dict(name="att_8b_bf16", seed=102, B=3, Hq=32, Hkv=8, D=128, S=16, P=16,
         ctx=[1, 17, 100], dtype="bf16"),
    # Qwen3-30B-A3B head shape (bf16, G = 8)
    dict(name="att_moe_bf16", seed=103, B=2, Hq=32, Hkv=4, D=128, S=16, P=12,
         ctx=[33, 64], dtype="bf16"),
    # head_dim 64 with 32-token pages
    dict(name="att_d64_s32_bf16", seed=104, B=2, Hq=8, Hkv=2, D=64, S=32, P=8,
         ctx=[40, 64], dtype="bf16"),
    # the reference unit-test geometry: tiny head_dim, 3-token pages, MHA
    dict(name="att_small_f32", seed=105, B=2, Hq=2, Hkv=2, D=8, S=3, P=5,
         ctx=[9, 4], dtype="f32"),
    # an empty request next to a non-empty one
    dict(name="att_empty_bf16", seed=106, B=2, Hq=8, Hkv=2, D=128, S=16, P=4,
         ctx=[0, 5], dtype="bf16"),
]


# Decode-prologue cases (QK-norm + RoPE of one new token per request): positions span
# the first token to 32k, where angles reach ~3e4 rad.
PROLOGUE_CASES = [
    # Qwen3-8B head shape, dense runner (no QK-norm), theta 1e6
    dict(name="pro_8b", seed=201, B=6, Hq=32, Hkv=8, D=128, base=1e6, qk_norm=False,
         positions=[0, 1, 511, 4095, 8191, 32767]),
    # Qwen3-30B-A3B head shape with QK-norm (MoE runner)
    dict(name="pro_moe_qk", seed=202, B=5, Hq=32, Hkv=4, D=128, base=1e6, qk_norm=True,
         positions=[3, 100, 2047, 4096, 30000]),
    # C1 shape (head_dim 64)
    dict(name="pro_c1", seed=203, B=4, Hq=4, Hkv=2, D=64, base=1e6, qk_norm=False,
         positions=[7, 22, 47, 63]),
    # head_dim 256, theta 1e4, QK-norm
    dict(name="pro_d256_qk", seed=204, B=3, Hq=8, Hkv=2, D=256, base=1e4, qk_norm=True,
         positions=[0, 777, 16383]),
]


# Prefill cases for _attn_paged (one request, q_len new tokens after q_start):
# q_start == 0 / non-causal go through its is_causal SDPA path, q_start > 0 through its
# dense offset mask. fp32 (the reference's exact path).
PREFILL_CASES = [
    dict(name="pf_causal0", seed=301, q_len=37, kv_len=37, q_start=0, causal=True,
         Hq=4, Hkv=2, D=64, S=16),
    dict(name="pf_offset", seed=302, q_len=13, kv_len=33, q_start=20, causal=True,
         Hq=8, Hkv=2, D=64, S=16),
    dict(name="pf_noncausal", seed=303, q_len=9, kv_len=40, q_start=31, causal=False,
         Hq=4, Hkv=4, D=64, S=16),
    dict(name="pf_g8_d128", seed=304, q_len=11, kv_len=17, q_start=6, causal=True,
         Hq=16, Hkv=2, D=128, S=16),
]


# host_stream_attention_v1 cases: a contiguous KV of `total` tokens split into host
# chunks of `chunk` tokens ([H_kv, D, C], the reference's host layout) covering the first
# `host` tokens, plus the resident tail. The first four follow the shapes of the
# reference's own tests of the op; the rest are model-sized. fp32 ~ 0.3 N(0, 1).
HOST_STREAM_CASES = [
    dict(name="hs_tail_prefill", seed=401, total=10, host=6, chunk=3, q_len=2, q_start=10,
         causal=True, Hq=4, Hkv=2, D=16),
    dict(name="hs_decode", seed=402, total=8, host=5, chunk=4, q_len=1, q_start=8,
         causal=True, Hq=4, Hkv=2, D=16),
    dict(name="hs_offset_suffix", seed=403, total=8, host=4, chunk=2, q_len=2, q_start=5,
         causal=True, Hq=4, Hkv=2, D=16),
    dict(name="hs_all_resident", seed=404, total=6, host=0, chunk=3, q_len=6, q_start=0,
         causal=True, Hq=4, Hkv=2, D=16),
    dict(name="hs_8b_decode", seed=405, total=700, host=640, chunk=64, q_len=1, q_start=700,
         causal=True, Hq=32, Hkv=8, D=128),
    dict(name="hs_moe_suffix", seed=406, total=300, host=256, chunk=128, q_len=5, q_start=295,
         causal=True, Hq=32, Hkv=4, D=128),
    dict(name="hs_noncausal", seed=407, total=90, host=60, chunk=20, q_len=3, q_start=0,
         causal=False, Hq=8, Hkv=8, D=64),
]


def host_stream_inputs(case: dict) -> dict:
    """q [1, q_len, Hq, D]; host chunks (k_c, v_c) [H_kv, D, C]; resident [1, R, H_kv, D]."""
    rng = np.random.default_rng(case["seed"])
    Hkv, D = case["Hkv"], case["D"]
    k_full = (0.3 * rng.standard_normal((1, case["total"], Hkv, D))).astype(np.float32)
    v_full = (0.3 * rng.standard_normal((1, case["total"], Hkv, D))).astype(np.float32)
    q = (0.3 * rng.standard_normal((1, case["q_len"], case["Hq"], D))).astype(np.float32)
    chunks = []
    for s in range(0, case["host"], case["chunk"]):
        e = min(s + case["chunk"], case["host"])
        chunks.append((np.ascontiguousarray(k_full[0, s:e].transpose(1, 2, 0)),
                       np.ascontiguousarray(v_full[0, s:e].transpose(1, 2, 0))))
    return dict(q=q, chunks=chunks, rk=np.ascontiguousarray(k_full[:, case["host"]:]),
                rv=np.ascontiguousarray(v_full[:, case["host"]:]), k_full=k_full, v_full=v_full)


def prefill_inputs(case: dict) -> dict:
    """q [q_len, Hq, D] and the context's K/V rows [kv_len, Hkv, D], float32 ~N(0,1)."""
    rng = np.random.default_rng(case["seed"])
    return dict(q=rng.standard_normal((case["q_len"], case["Hq"], case["D"]), dtype=np.float32),
                k=rng.standard_normal((case["kv_len"], case["Hkv"], case["D"]), dtype=np.float32),
                v=rng.standard_normal((case["kv_len"], case["Hkv"], case["D"]), dtype=np.float32))


def prologue_inputs(case: dict) -> dict:
    """q [B,Hq,D], k / v [B,Hkv,D] float32 ~N(0,1); QK-norm weights ~1 + 0.1 N(0,1)."""
    rng = np.random.default_rng(case["seed"])
    B, Hq, Hkv, D = (case[k] for k in ("B", "Hq", "Hkv", "D"))
    out = dict(q=rng.standard_normal((B, Hq, D), dtype=np.float32),
               k=rng.standard_normal((B, Hkv, D), dtype=np.float32),
               v=rng.standard_normal((B, Hkv, D), dtype=np.float32),
               positions=np.asarray(case["positions"], dtype=np.int64))
    if case["qk_norm"]:
        out["q_norm_w"] = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
        out["k_norm_w"] = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    return out


def attention_inputs(case: dict) -> dict:
    """q [B,Hq,D], logical pools [P,Hkv,D,S] (float32 values; bf16-representable for
    bf16 cases, plus their bit patterns) and block tables of distinct random pages."""
    rng = np.random.default_rng(case["seed"])
    B, Hq, Hkv, D, S, P = (case[k] for k in ("B", "Hq", "Hkv", "D", "S", "P"))
    q = rng.standard_normal((B, Hq, D), dtype=np.float32)
    k = rng.standard_normal((P, Hkv, D, S), dtype=np.float32)
    v = rng.standard_normal((P, Hkv, D, S), dtype=np.float32)
    perm = rng.permutation(P)
    tables, cur = [], 0
    for n in case["ctx"]:
        npg = -(-n // S)
        tables.append([int(x) for x in perm[cur:cur + npg]])
        cur += npg
    assert cur <= P, "pool too small for the case"
    out = dict(q=q, k=k, v=v, tables=tables, ctx=list(case["ctx"]))
    if case["dtype"] == "bf16":
        for name in ("q", "k", "v"):
            bits = f32_to_bf16_bits(out[name])
            out[name + "_bits"] = bits
            out[name] = bf16_bits_to_f32(bits)
    return out


def checksum(*arrays: np.ndarray) -> float:
    return float(sum(np.asarray(a, dtype=np.float64).sum() for a in arrays))


# C1: tiny Qwen3-architecture dense decoder
C1_MODEL = dict(n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, hidden_dim=256,
                intermediate_dim=512, vocab_size=1024, max_seq_len=128, rope_base=1e6)
C1_SEED = 7
C1_DECODE_STEPS = 32
C1_LOGIT_STEPS = (0, 1, 2, 8, 16, 32)   # steps whose full logits are stored


def c1_weights() -> dict[str, np.ndarray]:
    """fp32 weights ~N(0, 0.02) from a seed; RMSNorm weights are 1."""
    m = C1_MODEL
    rng = np.random.default_rng(C1_SEED)
    hid, inter, voc = m["hidden_dim"], m["intermediate_dim"], m["vocab_size"]
    qd = m["n_heads"] * m["head_dim"]
    kvd = m["n_kv_heads"] * m["head_dim"]

    def w(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)

    ws = {"embed_tokens.weight": w(voc, hid)}
    for i in range(m["n_layers"]):
        p = f"layers.{i}."
        ws[p + "input_layernorm.weight"] = np.ones(hid, np.float32)
        ws[p + "self_attn.q_proj.weight"] = w(qd, hid)
        ws[p + "self_attn.k_proj.weight"] = w(kvd, hid)
        ws[p + "self_attn.v_proj.weight"] = w(kvd, hid)
        ws[p + "self_attn.o_proj.weight"] = w(hid, qd)
        ws[p + "post_attention_layernorm.weight"] = np.ones(hid, np.float32)
        ws[p + "mlp.gate_proj.weight"] = w(inter, hid)
        ws[p + "mlp.up_proj.weight"] = w(inter, hid)
        ws[p + "mlp.down_proj.weight"] = w(hid, inter)
    ws["norm.weight"] = np.ones(hid, np.float32)
    ws["lm_head.weight"] = w(voc, hid)
    return ws


def c1_prompts() -> list[list[int]]:
    """4 prompts with lengths uniform in [8, 64], token ids uniform in [0, vocab)."""
    rng = np.random.default_rng(C1_SEED + 1)
    lens = rng.integers(8, 65, size=4)
    return [[int(t) for t in rng.integers(0, C1_MODEL["vocab_size"], size=int(n))] for n in lens]


# Index-copy / host-store scenario inputs
def token_kv(seed: int, n_tokens: int, n_layers: int, n_heads: int, head_dim: int,
             dtype: str) -> tuple[np.ndarray, np.ndarray]:
    """Per-token K/V [n_tokens, L, H, D]; float32 values (bf16-representable for bf16)."""
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((n_tokens, n_layers, n_heads, head_dim), dtype=np.float32)
    v = rng.standard_normal((n_tokens, n_layers, n_heads, head_dim), dtype=np.float32)
    if dtype == "bf16":
        k = bf16_bits_to_f32(f32_to_bf16_bits(k))
        v = bf16_bits_to_f32(f32_to_bf16_bits(v))
    return k, v
