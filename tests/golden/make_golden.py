"""Generate golden vectors by running the reference plastic-infer itself on CPU.

Run from the repository root, with the reference source tree available:

    python tests/golden/make_golden.py --ref <path-to-plastic-infer>/src

It imports the reference package read-only (no bytecode is written into its
tree), runs the reference's own functions on seeded inputs from
tests/golden/inputs.py, and writes small fixtures next to this file:

  index_copy_{bf16,f32}.npz   KVRequestCache.append_token + _write_kv_layer results
  attention.npz               paged_attention_v1 outputs for every ATTENTION_CASES entry
  store_{f32,bf16}.npz        sink_completed_chunks / load_prefix results
  chunk_keys.json             compute_prefix_hashes outputs
  allocator.json              PageAllocator alloc/free traces
  c1_tiny.npz                 prefill_forward_paged + 32 decode_step_paged greedy steps (C1)
  prologue.npz                qk_norm + rope_positions (fp32 table of build_rope_cache) outputs
                              for every PROLOGUE_CASES entry
  prefill.npz                 _attn_paged prefill outputs (is_causal, offset mask, non-causal)
                              and the block tables the reference's allocator produced

The fixtures are what the oracle is pinned against (tests/test_oracle_golden.py)
and what the GPU parity tests compare with; the reference tree itself is never
needed at test time.
"""

from __future__ import annotations

import argparse
import json
import os
import pathlib
import sys

sys.dont_write_bytecode = True
os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from tests.golden.inputs import (  # noqa: E402
    ATTENTION_CASES, C1_DECODE_STEPS, C1_LOGIT_STEPS, C1_MODEL, HOST_STREAM_CASES, PREFILL_CASES,
    PROLOGUE_CASES, attention_inputs, c1_prompts, c1_weights, checksum, host_stream_inputs,
    prefill_inputs, prologue_inputs, token_kv,
)
from oracle.paged_kv_oracle import f32_to_bf16_bits  # noqa: E402


def _bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    return t.contiguous().numpy().copy()


def _to_torch(a: np.ndarray, dtype: str) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    return t.to(torch.bfloat16) if dtype == "bf16" else t


def gen_index_copy(ref, dtype: str) -> None:
    KVConfig, KVStore = ref["KVConfig"], ref["KVStore"]
    write_kv_layer = ref["_write_kv_layer"]
    if dtype == "bf16":
        L, H, D, S, P, ntok = 2, 2, 64, 16, 12, 40
        tdt = torch.bfloat16
    else:
        L, H, D, S, P, ntok = 2, 2, 4, 4, 64, 20
        tdt = torch.float32
    cfg = KVConfig(n_layers=L, n_kv_heads=H, head_dim=D, page_size=S, pages_per_chunk=2,
                   max_pages=P, dtype=tdt, device=torch.device("cpu"))
    store = KVStore(cfg)
    caches = [store.new_request(), store.new_request()]
    k, v = token_kv(11 if dtype == "bf16" else 12, ntok, L, H, D, dtype)
    slots, kn, vn = [], [], []
    for t in range(ntok):
        cache = caches[0] if t % 3 else caches[1]   # interleave -> non-contiguous pages
        pos = cache.length
        cache.append_token(_to_torch(k[t], dtype), _to_torch(v[t], dtype))
        for layer in range(L):
            slots.append(cache.block_table.get_page(layer, pos // S) * S + pos % S)
            kn.append(k[t, layer])
            vn.append(v[t, layer])
    # Overwrite part of request 0 through the prefill-path writer (_write_kv_layer).
    c0 = caches[0]
    start, T = 2, min(7, c0.length - 2)
    k2, v2 = token_kv(13, T, 1, H, D, dtype)
    for layer in range(L):
        kt = _to_torch(k2[:, 0], dtype).unsqueeze(0) * (layer + 1)
        vt = _to_torch(v2[:, 0], dtype).unsqueeze(0) * (layer + 1)
        write_kv_layer(c0, store, layer, start, kt, vt)
        for t in range(T):
            pos = start + t
            slots.append(c0.block_table.get_page(layer, pos // S) * S + pos % S)
            kn.append(kt[0, t].float().numpy())
            vn.append(vt[0, t].float().numpy())
    kn = np.stack(kn).astype(np.float32)
    vn = np.stack(vn).astype(np.float32)
    out = dict(slots=np.asarray(slots, np.int64), page_size=S, num_pages=P, n_layers=L)
    if dtype == "bf16":
        out.update(k_new=f32_to_bf16_bits(kn), v_new=f32_to_bf16_bits(vn),
                   k_pages=_bits(store.gpu.k_pages), v_pages=_bits(store.gpu.v_pages))
    else:
        out.update(k_new=kn, v_new=vn, k_pages=_bits(store.gpu.k_pages),
                   v_pages=_bits(store.gpu.v_pages))
    np.savez_compressed(HERE / f"index_copy_{dtype}.npz", **out)


def gen_attention(ref) -> None:
    paged_attention_v1 = ref["paged_attention_v1"]
    out = {}
    for case in ATTENTION_CASES:
        x = attention_inputs(case)
        kp = torch.from_numpy(x["k"])
        vp = torch.from_numpy(x["v"])
        res = []
        for b in range(case["B"]):
            qb = torch.from_numpy(x["q"][b])[None, None]
            o = paged_attention_v1(qb, kp, vp, x["tables"][b], case["S"],
                                   kv_num_tokens=x["ctx"][b], causal=False)
            res.append(o[0, 0].numpy())
        r = np.stack(res).astype(np.float32)
        out[case["name"] + "/out"] = np.nan_to_num(r, nan=0.0)
        out[case["name"] + "/nan_mask"] = np.isnan(r)
        out[case["name"] + "/checksum"] = np.float64(checksum(x["q"], x["k"], x["v"]))
    np.savez_compressed(HERE / "attention.npz", **out)


def gen_store(ref, dtype: str) -> None:
    KVConfig, KVStore = ref["KVConfig"], ref["KVStore"]
    if dtype == "f32":
        L, H, D, S, ppc, P, tdt = 2, 2, 4, 4, 2, 64, torch.float32
    else:
        L, H, D, S, ppc, P, tdt = 2, 2, 64, 16, 2, 32, torch.bfloat16
    cfg = KVConfig(n_layers=L, n_kv_heads=H, head_dim=D, page_size=S, pages_per_chunk=ppc,
                   max_pages=P, max_host_chunks=8, dtype=tdt, device=torch.device("cpu"))
    store = KVStore(cfg)
    chunk = S * ppc
    ntok = 2 * chunk + chunk // 2
    k, v = token_kv(21 if dtype == "f32" else 22, ntok, L, H, D, dtype)
    rng = np.random.default_rng(23)
    tokens = [int(t) for t in rng.integers(0, 50000, size=ntok)]
    c1 = store.new_request()
    for t in range(ntok):
        c1.append_token(_to_torch(k[t], dtype), _to_torch(v[t], dtype))
    c1.set_token_ids(tokens)
    sunk = store.sink_completed_chunks(c1)
    host_k = np.stack([_bits(store._host_cache[key.full_key][0]) for key in c1.chunk_keys])
    host_v = np.stack([_bits(store._host_cache[key.full_key][1]) for key in c1.chunk_keys])
    keys_hex = [key.full_key.hex() for key in c1.chunk_keys]
    c1_tables = np.asarray([c1.get_block_table_for_layer(layer) for layer in range(L)], np.int64)
    store.free_request(c1)
    c2 = store.new_request()
    matched, _ = store.load_prefix(c2, tokens)
    c2_tables = np.asarray([c2.get_block_table_for_layer(layer) for layer in range(L)], np.int64)
    loaded_k = np.stack([_bits(store.gpu.k_pages[c2_tables[layer]]) for layer in range(L)])
    loaded_v = np.stack([_bits(store.gpu.v_pages[c2_tables[layer]]) for layer in range(L)])
    np.savez_compressed(
        HERE / f"store_{dtype}.npz",
        tokens=np.asarray(tokens, np.int64), sunk=sunk, host_k=host_k, host_v=host_v,
        keys_hex=np.asarray(keys_hex), c1_tables=c1_tables, c2_tables=c2_tables,
        matched=matched, c2_length=c2.length, loaded_k=loaded_k, loaded_v=loaded_v,
        free_after_load=store.gpu.allocator.free_pages,
        L=L, H=H, D=D, S=S, ppc=ppc, P=P,
    )


def gen_chunk_keys(ref) -> None:
    compute = ref["compute_prefix_hashes"]
    rng = np.random.default_rng(31)
    cases = {
        "range16_c8": (list(range(16)), 8),
        "rand512_c256": ([int(t) for t in rng.integers(0, 151936, size=512)], 256),
        "maxu32_c4": ([0xFFFFFFFF, 0, 1, 0x80000000] * 3, 4),
        "empty_c8": ([], 8),
    }
    out = {}
    for name, (toks, cs) in cases.items():
        keys = compute(toks, chunk_size=cs)
        out[name] = dict(tokens=toks, chunk_size=cs,
                         prefix=[k.prefix_key.hex() for k in keys],
                         cumulative=[k.cumulative_key.hex() for k in keys])
    (HERE / "chunk_keys.json").write_text(json.dumps(out, indent=1))


def gen_allocator(ref) -> None:
    PageAllocator = ref["PageAllocator"]
    a = PageAllocator(10)
    trace = []
    ops = [("alloc",), ("alloc",), ("alloc",), ("free", 1), ("alloc",), ("alloc_many", 4),
           ("free_many", [0, 3, 4]), ("alloc",), ("alloc_many", 3), ("free", 2), ("alloc",)]
    for op in ops:
        if op[0] == "alloc":
            r = a.alloc()
        elif op[0] == "alloc_many":
            r = a.alloc_many(op[1])
        elif op[0] == "free":
            r = a.free(op[1])
        else:
            r = a.free_many(op[1])
        trace.append(dict(op=list(op), result=r, free=a.free_pages, used=a.used_pages))
    (HERE / "allocator.json").write_text(json.dumps(trace, indent=1))


def gen_c1(ref) -> None:
    ModelConfig, DenseWeights = ref["ModelConfig"], ref["DenseWeights"]
    prefill, decode = ref["prefill_forward_paged"], ref["decode_step_paged"]
    make_kv_config, KVStore = ref["make_kv_config"], ref["KVStore"]
    cfg = ModelConfig(**C1_MODEL, dtype=torch.float32)
    weights = DenseWeights({k: torch.from_numpy(v) for k, v in c1_weights().items()})
    prompts = c1_prompts()
    kv_cfg = make_kv_config(cfg, max_pages=256, max_host_chunks=8)
    store = KVStore(kv_cfg)
    tokens, logits_keep, margins = [], [], []
    for prompt in prompts:
        cache = store.new_request()
        lg = prefill(weights, cfg, store, cache, torch.tensor(prompt))
        seq, keep, marg = [], [], []
        for step in range(C1_DECODE_STEPS + 1):
            if step > 0:
                lg = decode(weights, cfg, store, cache, seq[-1])
            top2 = torch.topk(lg, 2).values
            marg.append(float(top2[0] - top2[1]))
            seq.append(int(lg.argmax()))
            if step in C1_LOGIT_STEPS:
                keep.append(lg.numpy().copy())
        tokens.append(seq)
        logits_keep.append(np.stack(keep))
        margins.append(marg)
    np.savez_compressed(
        HERE / "c1_tiny.npz",
        prompt_lens=np.asarray([len(p) for p in prompts], np.int64),
        prompts=np.concatenate([np.asarray(p, np.int64) for p in prompts]),
        tokens=np.asarray(tokens, np.int64),
        logits=np.stack(logits_keep).astype(np.float32),
        logit_steps=np.asarray(C1_LOGIT_STEPS, np.int64),
        margins=np.asarray(margins, np.float64),
    )


def gen_prologue(ref) -> None:
    """qk_norm + rope_positions of the reference on one new token per request.

    The reference applies rope_positions to [batch, seq, heads, D] with one position per
    seq index; B requests with one token each are passed as seq = B. The table is
    build_rope_cache's fp32 one. inv_freq is stored as that function computes it
    (attention.py:68), and checked to reproduce the table's cos column by column.
    """
    build_rope_cache, rope_positions, qk_norm = (ref["build_rope_cache"], ref["rope_positions"],
                                                 ref["qk_norm"])
    out = {}
    for case in PROLOGUE_CASES:
        x = prologue_inputs(case)
        D, base = case["D"], case["base"]
        pos = torch.from_numpy(x["positions"])
        cos, sin = build_rope_cache(int(pos.max()) + 1, D, base=base, dtype=torch.float32)
        inv = 1.0 / (base ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
        freqs = torch.outer(torch.arange(int(pos.max()) + 1, dtype=torch.float32), inv)
        assert torch.equal(cos, torch.cat((freqs, freqs), dim=-1).cos())
        q = torch.from_numpy(x["q"])[None]
        k = torch.from_numpy(x["k"])[None]
        if case["qk_norm"]:
            q, k = qk_norm(q, k, torch.from_numpy(x["q_norm_w"]), torch.from_numpy(x["k_norm_w"]), D)
        qr = rope_positions(cos, sin, pos, q)[0]
        kr = rope_positions(cos, sin, pos, k)[0]
        n = case["name"]
        out[f"{n}__q"] = qr.numpy().copy()
        out[f"{n}__k"] = kr.numpy().copy()
        out[f"{n}__inv_freq"] = inv.numpy().copy()
        out[f"{n}__checksum"] = np.float64(checksum(*(x[k_] for k_ in sorted(x))))
    np.savez_compressed(HERE / "prologue.npz", **out)


def gen_prefill(ref) -> None:
    """_attn_paged on a KVStore filled token by token with append_token (fp32, CPU)."""
    KVConfig, KVStore, attn_paged = ref["KVConfig"], ref["KVStore"], ref["_attn_paged"]
    out = {}
    for case in PREFILL_CASES:
        x = prefill_inputs(case)
        S, Hkv, D, kv = case["S"], case["Hkv"], case["D"], case["kv_len"]
        cfg = KVConfig(n_layers=1, n_kv_heads=Hkv, head_dim=D, page_size=S, pages_per_chunk=2,
                       max_pages=-(-kv // S) + 3, dtype=torch.float32, device=torch.device("cpu"))
        store = KVStore(cfg)
        cache = store.new_request()
        for t in range(kv):
            cache.append_token(torch.from_numpy(x["k"][t])[None], torch.from_numpy(x["v"][t])[None])
        q = torch.from_numpy(x["q"])[None]
        o = attn_paged(q, cache, 0, store, kv_num_tokens=kv, causal=case["causal"],
                       q_start_pos=case["q_start"])
        n = case["name"]
        out[f"{n}__out"] = o[0].numpy().copy()
        out[f"{n}__table"] = np.asarray(cache.get_block_table_for_layer(0), dtype=np.int32)
        out[f"{n}__checksum"] = np.float64(checksum(x["q"], x["k"], x["v"]))
    np.savez_compressed(HERE / "prefill.npz", **out)


def gen_host_stream(ref) -> None:
    """host_stream_attention_v1 on CPU fp32 tensors, host chunks in the reference layout."""
    hs = ref["host_stream_attention_v1"]
    out = {}
    for case in HOST_STREAM_CASES:
        x = host_stream_inputs(case)
        chunks = [(torch.from_numpy(kc), torch.from_numpy(vc)) for kc, vc in x["chunks"]]
        o = hs(torch.from_numpy(x["q"]), chunks, torch.from_numpy(x["rk"]),
               torch.from_numpy(x["rv"]), q_start_pos=case["q_start"], causal=case["causal"])
        n = case["name"]
        out[f"{n}__out"] = o.numpy().copy()
        out[f"{n}__checksum"] = np.float64(checksum(x["q"], x["k_full"], x["v_full"]))
    np.savez_compressed(HERE / "host_stream.npz", **out)


def load_reference(src: str) -> dict:
    sys.path.insert(0, src)
    from plastic_infer.exec.attention import (
        build_rope_cache, host_stream_attention_v1, paged_attention_v1, qk_norm, rope_positions,
    )
    from plastic_infer.exec.runner import DenseWeights, ModelConfig
    from plastic_infer.exec.runner_paged import (
        _attn_paged, _write_kv_layer, decode_step_paged, make_kv_config, prefill_forward_paged,
    )
    from plastic_infer.kv.chunk import compute_prefix_hashes
    from plastic_infer.kv.kv_store import KVConfig, KVStore
    from plastic_infer.kv.paged import PageAllocator
    return dict(locals())


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path to the reference's src/ directory")
    ap.add_argument("--only", nargs="*", default=None,
                    help="generate only these fixtures (index_copy, attention, store, "
                         "chunk_keys, allocator, c1, prologue, prefill, host_stream)")
    args = ap.parse_args()
    torch.manual_seed(0)
    ref = load_reference(args.ref)
    gens = dict(
        index_copy=lambda: (gen_index_copy(ref, "bf16"), gen_index_copy(ref, "f32")),
        attention=lambda: gen_attention(ref),
        store=lambda: (gen_store(ref, "f32"), gen_store(ref, "bf16")),
        chunk_keys=lambda: gen_chunk_keys(ref),
        allocator=lambda: gen_allocator(ref),
        c1=lambda: gen_c1(ref),
        prologue=lambda: gen_prologue(ref),
        prefill=lambda: gen_prefill(ref),
        host_stream=lambda: gen_host_stream(ref),
    )
    for name, gen in gens.items():
        if args.only is None or name in args.only:
            gen()
    for p in sorted(HERE.glob("*.npz")) + sorted(HERE.glob("*.json")):
        print(f"{p.name:28s} {p.stat().st_size:9d} B")


if __name__ == "__main__":
    main()
