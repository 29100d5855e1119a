"""Benchmark of the paged-KV decode hot path on B200 (one JSON line on rank 0).

Workload ("C3"): one decode step of a Qwen3-8B-shape model's KV
path for a batch of 64 requests with ragged contexts uniform in [512, 8192]:
for each of 36 layers, the slot-mapping index-copy of the step's 64 new K/V rows
followed by paged GQA decode attention (32 query / 8 KV heads, head_dim 128, 16-token
pages, bf16) over every request's whole context. Every layer has its own block
tables of random, non-contiguous pages in one global pool (as the reference's engine
lays out layers, src/plastic_infer/runtime/engine.py:501-507), so the ~41 GB of KV
read per step is far larger than L2 and no flush is needed. The model's projections
and MLP are outside the path and not run.

  value      decode tokens/s of the whole job (64 tokens per step), device time
  e2e        same through the public API with pinned host inputs/outputs: per step
             the H2D copy of q / new K,V / slot mapping / lengths and the D2H read of
             the attention outputs are inside the timed region
  roofline   the attention kernel: algorithmic bytes (context K/V + q + out + block
             table) / its CUDA-event time, against the measured HBM copy bandwidth
  c4         the C4 (Qwen3-30B-A3B shape) KV path on the same ranks: tok/s, its
             attention roofline and (N = 1) layer 0 of its timed step against the oracle
  c5         the C5 long-context decode through the KV store API on the same ranks (KV
             heads sharded, each rank streaming its own host chunks): tok/s, the
             host-link roofline and (rank 0) two (request, layer) outputs of the last step
             against the oracle over histories rebuilt from the host chunks and device
             pages; so every N of a scaling run records C3, C4 and C5
  index_copy C2 microbench (65536-page pool): GB/s at B = 1, 64, 512, a whole 36-layer
             step in one launch (2304) and a large-B sweep; graphs of back-to-back launches
             with L2 flushed before every timed replay
  cpu_baseline the oracle (numpy port of the reference path) on layer 0 of the timed step
  parity     that layer's GPU output against the oracle's (the run exits non-zero on a
             mismatch)

`--impl reference` times the reference's CPU path instead (rank 0 only): its own torch
operations (oracle/ref_torch_path.py), one real layer of the step per timed step.
Multi-GPU (torchrun, N = 2/4/8): KV heads and their pools are split across ranks;
each rank attends its heads and the per-layer outputs are all-gathered before o_proj
would run, inside the attention kernel (NVLink peer stores; --nccl: an NCCL
all-gather after it instead); time is the max over ranks, every rank's timed region
starting together on the device.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (Qwen3-8B shape, paged KV); index-copy GB/s vs HBM peak"
C3 = dict(layers=36, batch=64, hq=32, hkv=8, head_dim=128, page_size=16, ctx_lo=512,
          ctx_hi=8192, seed=0)
C2 = dict(pages=65536, page_size=16, hkv=8, head_dim=128,
          batches=(1, 64, 512, 2304, 4096, 65536))
C3["desc"] = ("C3 qwen3-8b-shape paged decode KV path: 36 layers x (index-copy of 64 new K/V "
              "rows + paged GQA decode attention), B=64, ctx U[512,8192] seed 0, 32q/8kv heads, "
              "head_dim 128, page 16")
# the attention/KV path of a Qwen3-30B-A3B-shape MoE decode step
# (the expert FFN is outside the path).
C4 = dict(layers=48, batch=128, hq=32, hkv=4, head_dim=128, page_size=16, ctx_lo=256,
          ctx_hi=4096, seed=0,
          desc="C4 qwen3-30b-a3b-shape paged decode KV path: 48 layers x (index-copy of 128 new "
               "K/V rows + paged GQA decode attention, G=8), B=128, ctx U[256,4096] seed 0, "
               "32q/4kv heads, head_dim 128, page 16",
          metric="decode tok/s (Qwen3-30B-A3B shape, paged KV attention path)")
# long-context offload. Device pool = 25% of all pages; the rest of
# every request's KV lives in the pinned host KV store (256-token chunks).
C5 = dict(layers=36, batch=8, hq=32, hkv=8, head_dim=128, page_size=16, pages_per_chunk=16,
          ctx=32768, pool_frac=0.25, seed=0)
WORKLOADS = {"c3": C3, "c4": C4}


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return dict(hbm_gbs=float(d["hbm_gbs"]), bf16_tflops=float(d.get("bf16_tflops", 1590.0)),
                    source="measured")
    return dict(hbm_gbs=6650.0, bf16_tflops=1590.0, source="fallback")


def c3_contexts(cfg: dict) -> np.ndarray:
    rng = np.random.default_rng(cfg["seed"])
    return rng.integers(cfg["ctx_lo"], cfg["ctx_hi"] + 1, size=cfg["batch"]).astype(np.int64)


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region.

    One sampler process per job (rank 0) covering every GPU of the job: `indices` are
    the local GPU indices to query (None: sample nothing).
    """

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, indices, interval_ms: int = 20) -> None:
        self.indices = indices
        self.interval_ms = interval_ms
        self.proc = None
        self.out = ""
        self.first = ""

    def __enter__(self):
        if not self.indices:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ",".join(map(str, self.indices)), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", str(self.interval_ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            # nvidia-smi needs a moment to start; the first line marks it sampling
            self.first = self.proc.stdout.readline()
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc) -> None:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self) -> dict:
        rows = []
        for line in (self.out or "").splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                rows.append(parts)
        if not rows:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=["unsampled"], samples=0)
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[3 + i] == "Active"})
        return dict(sm_mhz=statistics.median(sm) if sm else None,
                    sm_max_mhz=float(rows[0][1]) if rows[0][1].replace(".", "").isdigit() else None,
                    reasons=reasons, samples=len(rows))


# ---------------------------------------------------------------------------------
# C3 decode step on the device
# ---------------------------------------------------------------------------------


class DecodeWorkload:
    """Device state of one C3 decode step for this rank's KV-head shard."""

    def __init__(self, cfg: dict, rank: int, world: int, dev: torch.device) -> None:
        from plastic_infer_b200 import kernels

        self.kernels = kernels
        self.cfg = cfg
        from plastic_infer_b200.dist import head_shard

        L, B, S, D = cfg["layers"], cfg["batch"], cfg["page_size"], cfg["head_dim"]
        # This rank's KV heads and query heads; with fewer KV heads than ranks (C4 on 8
        # GPUs) each KV head is replicated and its replicas split its query heads.
        self.shard = head_shard(cfg["hq"], cfg["hkv"], world, rank)
        self.hkv = self.shard.n_kv
        self.hq = self.shard.n_q
        self.dev = dev
        self.ctx = c3_contexts(cfg)
        npg = (self.ctx + S - 1) // S
        self.pages_per_layer = int(npg.sum())
        self.total_pages = self.pages_per_layer * L
        maxp = int(npg.max())
        # Block tables: every layer draws its pages from one global random permutation
        # (identical on every rank: page ids are replicated, pools are head-sharded).
        rng = np.random.default_rng(cfg["seed"] + 1)
        perm = rng.permutation(self.total_pages).astype(np.int32)
        bt = np.zeros((L, B, maxp), np.int32)
        cur = 0
        for l in range(L):
            for b in range(B):
                bt[l, b, :npg[b]] = perm[cur:cur + npg[b]]
                cur += npg[b]
        self.block_tables = torch.from_numpy(bt).to(dev)
        last = self.ctx - 1
        slots = bt[np.arange(L)[:, None], np.arange(B)[None, :], last[None, :] // S] * S + last % S
        self.slots_host = torch.from_numpy(slots.astype(np.int64)).pin_memory()
        self.ctx_host = torch.from_numpy(self.ctx.astype(np.int32)).pin_memory()
        self.slots = self.slots_host.to(dev)
        self.ctx_lens = self.ctx_host.to(dev)
        shape = (self.total_pages, self.hkv, S, D)
        g = torch.Generator(device=dev).manual_seed(1234 + rank)
        self.k_pool = torch.empty(shape, dtype=torch.bfloat16, device=dev).normal_(generator=g)
        self.v_pool = torch.empty(shape, dtype=torch.bfloat16, device=dev).normal_(generator=g)
        self.q = torch.randn((L, B, self.hq, D), dtype=torch.bfloat16, device=dev, generator=g)
        self.k_new = torch.randn((L, B, self.hkv, D), dtype=torch.bfloat16, device=dev, generator=g)
        self.v_new = torch.randn((L, B, self.hkv, D), dtype=torch.bfloat16, device=dev, generator=g)
        self.out = torch.empty((L, B, self.hq, D), dtype=torch.bfloat16, device=dev)
        self.ws = kernels.Workspace(dev)
        self.world = world
        self.fused = False
        self.gathered = None
        self.exchange = None
        if world > 1:
            # rank-major [world * B, Hq/N, D] per layer (what o_proj would consume)
            self.gathered = torch.empty((L, world * B, self.hq, D), dtype=torch.bfloat16, device=dev)

    def use_peer_gather(self) -> None:
        """Gather through the kernel's NVLink peer stores (one slot per layer)."""
        from plastic_infer_b200.dist import PeerExchange

        if self.cfg["layers"] < 3:
            raise SystemExit("the peer all-gather path needs at least 3 layers (output slots)")
        self.exchange = PeerExchange(self.cfg["batch"], self.hq, self.cfg["head_dim"],
                                     torch.bfloat16, slots=self.cfg["layers"])

    # algorithmic bytes of one attention launch (one layer) for this rank
    def attn_bytes(self) -> float:
        D, B = self.cfg["head_dim"], self.cfg["batch"]
        kv = float(self.ctx.sum()) * self.hkv * D * 2 * 2
        qo = 2.0 * B * self.hq * D * 2
        tables = 4.0 * self.pages_per_layer + 4.0 * B
        return kv + qo + tables

    def copy_bytes(self) -> float:
        # one index-copy launch: B tokens x (K+V) x (read + write) rows + slot ids
        return float(self.cfg["batch"]) * (2 * 2 * self.hkv * self.cfg["head_dim"] * 2 + 8)

    def layer(self, l: int, attention: bool = True, copy: bool = True, gather: bool = True) -> None:
        k = self.kernels
        if self.exchange is not None and attention and gather:
            # N > 1: attention with the all-gather fused in (NVLink peer stores; the
            # launch waits for every rank's previous launch before it starts)
            if copy:
                k.kv_index_copy(self.k_pool, self.v_pool, self.k_new[l], self.v_new[l],
                                self.slots[l])
            k.paged_decode_attention_gather(self.q[l], self.k_pool, self.v_pool,
                                            self.block_tables[l], self.ctx_lens, self.exchange,
                                            workspace=self.ws)
            return
        if attention and copy and self.fused:
            # one launch: write the 64 new K/V rows, then attend
            k.paged_decode_attention(self.q[l], self.k_pool, self.v_pool, self.block_tables[l],
                                     self.ctx_lens, out=self.out[l], workspace=self.ws,
                                     k_new=self.k_new[l], v_new=self.v_new[l],
                                     slot_mapping=self.slots[l])
        else:
            if copy:
                k.kv_index_copy(self.k_pool, self.v_pool, self.k_new[l], self.v_new[l],
                                self.slots[l])
            if attention:
                k.paged_decode_attention(self.q[l], self.k_pool, self.v_pool, self.block_tables[l],
                                         self.ctx_lens, out=self.out[l], workspace=self.ws)
        if self.world > 1 and gather:
            import torch.distributed as dist

            dist.all_gather_into_tensor(self.gathered[l], self.out[l])

    def step(self, attention: bool = True, copy: bool = True, gather: bool = True) -> None:
        for l in range(self.cfg["layers"]):
            self.layer(l, attention, copy, gather)


def time_region(fn, steps: int, stream: torch.cuda.Stream, world: int = 1) -> float:
    """Device ms for `steps` calls of fn, events on the launching stream.

    With several ranks a one-element all-reduce is queued right before the start
    event, so every rank's timed region starts when the last rank is ready (host-side
    skew before the region is not counted by the ranks that started early).
    """
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(torch.zeros(1, device=stream.device))
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end)


def graph_of(fn, warm: int = 1) -> torch.cuda.CUDAGraph:
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warm):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


class L2Flush:
    """Evicts L2 (126 MB on B200) between timed regions, outside them.

    A 256 MB buffer is written (evicting whatever was cached) and then read, so that L2
    is left holding clean lines: without the read, the written lines would still be
    dirty in L2 and their write-back would land inside the next timed region.
    """

    def __init__(self, dev: torch.device) -> None:
        self.buf = torch.empty(256 << 18, dtype=torch.int32, device=dev)
        self.sink = torch.empty((), dtype=torch.int64, device=dev)

    def __call__(self) -> None:
        self.buf.fill_(1)
        torch.sum(self.buf, dim=0, dtype=torch.int64, out=self.sink)


def bench_index_copy(dev: torch.device, peak: float) -> dict:
    """C2: scatter of B rows into a 65536-page bf16 pool; per-launch device time.

    Each B is timed as a CUDA graph of R back-to-back launches, as a decode step issues
    them (one per layer): launch i reads its own source rows and writes its own random
    distinct slots, and L2 is flushed (a 256 MB write then read, outside the timed
    region) before every timed replay, so no launch finds its rows in L2. B = 2304 is a whole
    36-layer step of the 8B shape written by one launch (all layers share the pool).
    """
    from plastic_infer_b200 import kernels

    P, S, H, D = C2["pages"], C2["page_size"], C2["hkv"], C2["head_dim"]
    g = torch.Generator(device=dev).manual_seed(7)
    kp = torch.zeros((P, H, S, D), dtype=torch.bfloat16, device=dev)
    vp = torch.zeros_like(kp)
    flush = L2Flush(dev)
    res = {}
    rng = np.random.default_rng(0)
    perm = torch.from_numpy(rng.permutation(P * S).astype(np.int64)).to(dev)
    for B in C2["batches"]:
        row_bytes = B * H * D * 2  # one of K or V
        R = int(max(8, min(100, (1 << 30) // row_bytes)))
        k_src = torch.randn((R, B, H, D), dtype=torch.bfloat16, device=dev, generator=g)
        v_src = torch.randn((R, B, H, D), dtype=torch.bfloat16, device=dev, generator=g)
        n_slots = P * S
        slots = torch.stack([perm[(i * B) % (n_slots - B + 1):][:B] for i in range(R)])

        def launches(k_src=k_src, v_src=v_src, slots=slots, R=R):
            for i in range(R):
                kernels.kv_index_copy(kp, vp, k_src[i], v_src[i], slots[i])

        graph = graph_of(launches)
        graph.replay()
        reps = 5
        ms = 0.0
        stream = torch.cuda.current_stream()
        for _ in range(reps):
            flush()
            ms += time_region(graph.replay, 1, stream)
        t = ms / (reps * R) * 1e-3
        byts = 8200.0 * B
        res[str(B)] = dict(us_per_launch=round(t * 1e6, 3), gbs=round(byts / t / 1e9, 1),
                           frac_of_hbm=round(byts / t / 1e9 / peak, 3), launches_per_graph=R)
        del graph, k_src, v_src, slots
    return res


def bench_page_copy(dev: torch.device, peak: float, profile: bool = False) -> dict:
    """Page gather / scatter between the pool and a chunk-layout staging buffer (row a3).

    The C5 sink unit: 8 chunks of 36 layers x 16 pages (4,608 pages, 151 MB per pool at
    the 8B head shape) at random ids of a 65,536-page bf16 pool, moved by one launch,
    as KVStore.sink_completed_chunks (gather) and load_prefix (scatter) issue them.
    Algorithmic bytes = 2 x the bytes moved (read + write). Timed as a CUDA graph of R
    back-to-back launches, each on its own random page set, with L2 flushed (write then
    read of 256 MB, outside the timed region) before every replay.
    """
    from plastic_infer_b200 import kernels

    P, S, H, D = C2["pages"], C2["page_size"], C2["hkv"], C2["head_dim"]
    n, R = 8 * 36 * 16, 6
    pool = torch.empty((P, H, S, D), dtype=torch.bfloat16, device=dev).normal_()
    staging = [torch.empty((n, H, S, D), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    rng = np.random.default_rng(3)
    ids = [torch.from_numpy(rng.permutation(P)[:n].astype(np.int32)).to(dev) for _ in range(R)]
    moved = float(staging[0].numel() * staging[0].element_size())
    flush = L2Flush(dev)
    stream = torch.cuda.current_stream()
    res = {}
    ops = {
        "gather": lambda i: kernels.page_gather(pool, ids[i], staging[i % 2], pages_per_group=16),
        "scatter": lambda i: kernels.page_scatter(staging[i % 2], ids[i], pool, pages_per_group=16),
    }
    for name, op in ops.items():
        if profile:
            for i in range(3):
                op(i)
            continue
        graph = graph_of(lambda op=op: [op(i) for i in range(R)])
        reps, ms = 5, 0.0
        for _ in range(reps):
            flush()
            ms += time_region(graph.replay, 1, stream)
        t = ms / (reps * R) * 1e-3
        res[name] = dict(us_per_launch=round(t * 1e6, 2), gbs=round(2 * moved / t / 1e9, 1),
                         frac_of_hbm=round(2 * moved / t / 1e9 / peak, 3), launches_per_graph=R)
        del graph
    torch.cuda.synchronize()
    return dict(workload=f"{n} pages (8 chunks x 36 layers x 16 pages) of a {P}-page bf16 pool, "
                         f"{H} heads x {S} x {D}; one launch", bytes_moved=int(moved),
                per_op=res, peak=peak)


def bench_prologue(dev: torch.device, peak: float) -> dict:
    """Fused decode prologue (QK-norm + RoPE + K/V slot write) per layer vs the unfused ops.

    The unfused sequence is what the reference's runners launch for the same work on the
    GPU (qk_norm, rope_positions on q and k over a model-dtype table, then the slot write,
    here our index-copy). Per-launch times from CUDA-graph replays of back-to-back steps.
    """
    from plastic_infer_b200 import kernels
    from plastic_infer_b200.exec.attention import build_rope_cache, qk_norm, rope_positions

    D, S, P = 128, 16, 4096
    shapes = {"c3": dict(B=64, Hq=32, Hkv=8, qk=False), "c4": dict(B=128, Hq=32, Hkv=4, qk=True)}
    res = {}
    g = torch.Generator(device=dev).manual_seed(21)
    for name, sh in shapes.items():
        B, Hq, Hkv, qk = sh["B"], sh["Hq"], sh["Hkv"], sh["qk"]
        q = torch.randn((B, Hq, D), dtype=torch.bfloat16, device=dev, generator=g)
        k = torch.randn((B, Hkv, D), dtype=torch.bfloat16, device=dev, generator=g)
        v = torch.randn((B, Hkv, D), dtype=torch.bfloat16, device=dev, generator=g)
        pos = torch.randint(0, 8192, (B,), device=dev, generator=g)
        slots = torch.randperm(P * S, device=dev, generator=g)[:B]
        kp = torch.zeros((P, Hkv, S, D), dtype=torch.bfloat16, device=dev)
        vp = torch.zeros_like(kp)
        qw = kw = None
        if qk:
            qw = 1 + 0.1 * torch.randn(D, device=dev, generator=g).to(torch.bfloat16)
            kw = 1 + 0.1 * torch.randn(D, device=dev, generator=g).to(torch.bfloat16)
        inv = kernels.rope_inv_freq(D, 1e6, dev)
        q_out = torch.empty_like(q)
        q_out2 = torch.empty_like(q)
        cos, sin = build_rope_cache(8192, D, base=1e6, device=dev, dtype=torch.bfloat16)

        def fused():
            kernels.decode_prologue(q, k, v, pos, inv, slots, kp, vp, qw, kw, q_out=q_out)

        def unfused():
            q4, k4 = q[None], k[None]  # one position per request: [1, B, heads, D]
            if qk:
                q4, k4 = qk_norm(q4, k4, qw, kw, D)
            kr = rope_positions(cos, sin, pos, k4)
            q_out2.copy_(rope_positions(cos, sin, pos, q4)[0])
            kernels.kv_index_copy(kp, vp, kr[0], v, slots)

        times = {}
        for label, fn in (("fused", fused), ("unfused", unfused)):
            graph = graph_of(fn)
            graph.replay()
            reps = 200
            times[label] = time_region(graph.replay, reps, torch.cuda.current_stream()) / reps * 1e3
            del graph
        byts = 2.0 * B * (Hq + 2 * Hkv) * D * 2 + 16.0 * B + 2.0 * D
        res[name] = dict(B=B, hq=Hq, hkv=Hkv, qk_norm=qk,
                         us_per_launch=round(times["fused"], 2),
                         unfused_us=round(times["unfused"], 2),
                         speedup=round(times["unfused"] / times["fused"], 2),
                         bytes_per_launch=int(byts),
                         gbs=round(byts / (times["fused"] * 1e-6) / 1e9, 1),
                         frac_of_hbm=round(byts / (times["fused"] * 1e-6) / 1e9 / peak, 4))
    return res


def bench_expert_copy(dev: torch.device) -> dict:
    """MoE expert-slot copy: the step's missing experts, host banks -> device slot caches.

    Qwen3-30B-A3B expert banks in bf16 (gate_up 2 x 768 x 2048, down 2048 x 768 per expert;
    128 experts of one layer in pinned host memory, 32 device slots). Ours against the
    reference's own fused multi-bank kernel (compiled from the reference tree into
    oracle/_ref/, when present) and against the host link's measured pinned copy rate.
    """
    from plastic_infer_b200 import kernels

    rows = (2 * 768 * 2048 * 2, 2048 * 768 * 2)  # bytes per expert row of each bank
    E, SL = 128, 32
    src = [torch.empty((E, rb), dtype=torch.uint8, pin_memory=True) for rb in rows]
    for t in src:
        t.random_(0, 256)
    dst = [torch.empty((SL, rb), dtype=torch.uint8, device=dev) for rb in rows]
    dptr = torch.tensor([d.data_ptr() for d in dst], dtype=torch.int64, device=dev)
    sptr = torch.tensor([x.data_ptr() for x in src], dtype=torch.int64, device=dev)
    feat = torch.tensor(list(rows), dtype=torch.int64, device=dev)
    # link peak: one pinned 1 GiB host->device copy
    h = torch.empty(1 << 30, dtype=torch.uint8, pin_memory=True)
    d = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
    d.copy_(h)
    torch.cuda.synchronize()
    link = (1 << 30) / (time_region(lambda: d.copy_(h, non_blocking=True), 3,
                                    torch.cuda.current_stream()) / 3 * 1e-3) / 1e9
    del h, d
    ref = None
    ref_path = os.path.join(ROOT, "oracle", "_ref", "libref_expert_copy.so")
    if os.path.exists(ref_path):
        import ctypes

        ref = ctypes.CDLL(ref_path)
        ref.ref_fast_index_copy_multi_launch.argtypes = [ctypes.c_void_p] * 5 + [
            ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        ref.ref_fast_index_copy_multi_launch.restype = None
    res = dict(link_gbs=round(link, 1), banks="gate_up 6.0 MiB + down 3.0 MiB per expert",
               reference_kernel="built" if ref is not None else "not built")
    rng = np.random.default_rng(5)
    for n in (1, 8, 32):
        di = torch.from_numpy(rng.permutation(SL)[:n].astype(np.int32)).to(dev)
        si = torch.from_numpy(rng.permutation(E)[:n].astype(np.int32)).to(dev)
        num = torch.tensor([n], dtype=torch.int64, device=dev)
        byts = float(n * sum(rows))

        def ours():
            kernels.expert_slot_copy(dptr, sptr, feat, di, si, num)

        def theirs():
            ref.ref_fast_index_copy_multi_launch(dptr.data_ptr(), sptr.data_ptr(), feat.data_ptr(),
                                                 di.data_ptr(), si.data_ptr(), n, num.data_ptr(),
                                                 len(rows), 1, torch.cuda.current_stream().cuda_stream)

        entry = {}
        for label, fn in (("ours", ours), ("reference_kernel", theirs)):
            if label == "reference_kernel" and ref is None:
                continue
            fn()
            torch.cuda.synchronize()
            reps = 20
            us = time_region(fn, reps, torch.cuda.current_stream()) / reps * 1e3
            entry[label] = dict(us=round(us, 1), gbs=round(byts / (us * 1e-6) / 1e9, 1),
                                frac_of_link=round(byts / (us * 1e-6) / 1e9 / link, 3))
        res[f"experts_{n}"] = dict(bytes=int(byts), **entry)
    return res


def bench_prefill(dev: torch.device, peaks: dict) -> dict:
    """Paged prefill attention of one request at the Qwen3-8B head shape (32 q / 8 KV heads,
    head_dim 128, 16-token pages, bf16): a first 4096-token prefill (causal from 0) and a
    1024-token chunk at position 3072 (the reference's offset-mask path). Ours against the
    reference's algorithm on the same GPU (page gather, repeat_interleave, SDPA with
    is_causal or with its dense mask). Ours is timed on both kernels: tcgen05 (S and O in
    tensor memory) and mma.sync. FLOPs = 4 * D * Hq * sum of the rows' key counts.
    """
    import torch.nn.functional as F

    from plastic_infer_b200 import kernels

    Hq, Hkv, D, S = 32, 8, 128, 16
    kv = 4096
    P = kv // S + 8
    g = torch.Generator(device=dev).manual_seed(31)
    kp = torch.randn((P, Hkv, S, D), dtype=torch.bfloat16, device=dev, generator=g)
    vp = torch.randn_like(kp)
    bt = torch.randperm(P, device=dev, generator=g)[:kv // S].to(torch.int32)
    res = {}
    for name, (q_len, q_start) in {"first_4096": (4096, 0), "chunk_1024_at_3072": (1024, 3072)}.items():
        q = torch.randn((q_len, Hq, D), dtype=torch.bfloat16, device=dev, generator=g)
        rows = torch.arange(q_start, q_start + q_len, dtype=torch.float64) + 1
        flops = 4.0 * D * Hq * float(rows.clamp(max=kv).sum())

        def ours_tc():
            kernels.paged_prefill_attention(q, kp, vp, bt, kv, q_start, True, impl="tc")

        def ours_mma():
            kernels.paged_prefill_attention(q, kp, vp, bt, kv, q_start, True, impl="mma")

        def reference():
            k = kp[bt.long()].permute(0, 2, 1, 3).reshape(-1, Hkv, D)[:kv]
            v = vp[bt.long()].permute(0, 2, 1, 3).reshape(-1, Hkv, D)[:kv]
            qt = q.transpose(0, 1)[None]
            kt = k.transpose(0, 1).repeat_interleave(Hq // Hkv, dim=0)[None]
            vt = v.transpose(0, 1).repeat_interleave(Hq // Hkv, dim=0)[None]
            if q_start == 0:
                return F.scaled_dot_product_attention(qt, kt, vt, is_causal=True)
            qpos = torch.arange(q_start, q_start + q_len, device=dev)
            mask = torch.arange(kv, device=dev)[None, :] <= qpos[:, None]
            am = torch.zeros(q_len, kv, dtype=q.dtype, device=dev).masked_fill(~mask, float("-inf"))
            return F.scaled_dot_product_attention(qt, kt, vt, attn_mask=am[None, None])

        entry = dict(q_len=q_len, q_start=q_start, kv_len=kv, gflop=round(flops / 1e9, 1))
        for label, fn in (("ours_tc", ours_tc), ("ours_mma", ours_mma),
                          ("reference_algorithm", reference)):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            reps = 10
            us = time_region(fn, reps, torch.cuda.current_stream()) / reps * 1e3
            entry[label] = dict(us=round(us, 1), tflops=round(flops / (us * 1e-6) / 1e12, 1))
        for label in ("ours_tc", "ours_mma"):
            entry[label]["speedup_vs_reference_algorithm"] = round(
                entry["reference_algorithm"]["us"] / entry[label]["us"], 2)
            entry[label]["frac_of_bf16_peak"] = round(entry[label]["tflops"] / peaks["bf16_tflops"], 3)
        res[name] = entry
    return res


def bench_host_stream(dev: torch.device) -> dict:
    """Host-stream decode attention at the C5 shape: 8 requests x 32768
    tokens, Qwen3-8B heads (32 q / 8 KV, head_dim 128), bf16. Each request's first 75% of
    tokens sit in pinned host chunks of 256 tokens ([H_kv, T, D], the KV store's chunk
    layout), the last 25% on the device. One step = one layer's decode attention of all
    8 requests.

    Ours reads the host chunks in place (pi_host_stream_attn). The reference's algorithm
    (host_stream_attention_v1: concatenate chunks + tail, repeat_interleave, SDPA) needs
    the chunks on the device first; it is timed with that host->device copy included
    (pinned, one cudaMemcpyAsync per chunk), on the same GPU. The bound is the host link:
    achieved = host bytes / time, against a pinned 1 GiB host->device copy measured here.
    """
    import torch.nn.functional as F

    from plastic_infer_b200 import kernels

    B, kv, Hq, Hkv, D, C = 8, 32768, 32, 8, 128, 256
    host_tok = kv * 3 // 4
    n_chunks = host_tok // C
    g = torch.Generator().manual_seed(51)
    h = torch.empty(1 << 30, dtype=torch.uint8, pin_memory=True)
    d = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
    d.copy_(h)
    torch.cuda.synchronize()
    link = (1 << 30) / (time_region(lambda: d.copy_(h, non_blocking=True), 3,
                                    torch.cuda.current_stream()) / 3 * 1e-3) / 1e9
    del h, d
    reqs = []
    for _ in range(B):
        kh = torch.randn((n_chunks, Hkv, C, D), generator=g).to(torch.bfloat16).pin_memory()
        vh = torch.randn((n_chunks, Hkv, C, D), generator=g).to(torch.bfloat16).pin_memory()
        kt = torch.randn((kv - host_tok, Hkv, D), device=dev, dtype=torch.bfloat16)
        vt = torch.randn((kv - host_tok, Hkv, D), device=dev, dtype=torch.bfloat16)
        q = torch.randn((1, Hq, D), device=dev, dtype=torch.bfloat16)
        spans = [(kh[i], vh[i]) for i in range(n_chunks)] + [(kt.permute(1, 0, 2), vt.permute(1, 0, 2))]
        reqs.append((kh, vh, kt, vt, q, spans))
    host_bytes = B * 2 * host_tok * Hkv * D * 2
    dev_bytes = B * 2 * (kv - host_tok) * Hkv * D * 2
    out = torch.empty((B, 1, Hq, D), device=dev, dtype=torch.bfloat16)

    def ours():
        for i, (_, _, _, _, q, spans) in enumerate(reqs):
            kernels.host_stream_attention(q, spans, q_start=kv - 1, out=out[i])

    stage_k = torch.empty((n_chunks, Hkv, C, D), device=dev, dtype=torch.bfloat16)
    stage_v = torch.empty_like(stage_k)

    def reference():
        for i, (kh, vh, kt, vt, q, _) in enumerate(reqs):
            for c in range(n_chunks):
                stage_k[c].copy_(kh[c], non_blocking=True)
                stage_v[c].copy_(vh[c], non_blocking=True)
            k = torch.cat([stage_k.permute(0, 2, 1, 3).reshape(-1, Hkv, D), kt])   # [kv, H, D]
            v = torch.cat([stage_v.permute(0, 2, 1, 3).reshape(-1, Hkv, D), vt])
            kt_ = k.transpose(0, 1).repeat_interleave(Hq // Hkv, dim=0)[None]
            vt_ = v.transpose(0, 1).repeat_interleave(Hq // Hkv, dim=0)[None]
            out[i] = F.scaled_dot_product_attention(q.transpose(0, 1)[None], kt_, vt_)[0].transpose(0, 1)

    res = dict(workload=f"C5 host-stream decode: {B} requests x {kv} tokens, {n_chunks} pinned "
                        f"host chunks of {C} tokens + {kv - host_tok}-token device tail per request, "
                        f"{Hq}q/{Hkv}kv heads, head_dim {D}, bf16; one layer",
               host_gb=round(host_bytes / 1e9, 3), device_gb=round(dev_bytes / 1e9, 3),
               link_gbs=round(link, 1))
    for label, fn in (("ours", ours), ("reference_algorithm", reference)):
        fn()
        torch.cuda.synchronize()
        reps = 3
        us = time_region(fn, reps, torch.cuda.current_stream()) / reps * 1e3
        res[label] = dict(us_per_layer=round(us, 1), host_gbs=round(host_bytes / (us * 1e-6) / 1e9, 1),
                          frac_of_link=round(host_bytes / (us * 1e-6) / 1e9 / link, 3))
    res["speedup"] = round(res["reference_algorithm"]["us_per_layer"] / res["ours"]["us_per_layer"], 2)
    return res


class LayerSnapshot:
    """Layer 0 of the timed step, copied on the device right after the timed region:
    the attention output and the pages it read (the step's new rows included)."""

    def __init__(self, wl: "DecodeWorkload") -> None:
        S = wl.cfg["page_size"]
        npg = (wl.ctx + S - 1) // S
        bt = wl.block_tables[0].cpu().numpy()
        ids = np.concatenate([bt[b, :npg[b]] for b in range(len(npg))]).astype(np.int64)
        dev_ids = torch.from_numpy(ids).to(wl.k_pool.device)
        self.k = wl.k_pool.index_select(0, dev_ids)
        self.v = wl.v_pool.index_select(0, dev_ids)
        self.out = wl.out[0].clone()
        self.q = wl.q[0].clone()
        self.k_new = wl.k_new[0].clone()
        self.v_new = wl.v_new[0].clone()
        self.ctx = wl.ctx.copy()
        self.npg = npg


class CpuSample:
    """The C3 KV path on the CPU with the oracle (a numpy port of the reference's
    _write_kv_layer + paged_attention_v1), run per layer on one layer's data.

    Built from a LayerSnapshot, the data are layer 0 of the step the GPU just timed
    (bf16 values widened to fp32, pools in the reference's logical [pages, Hkv, D, S]
    layout with the layer's pages renumbered 0..n-1), so the first layer the baseline
    runs is also the parity check of the timed step: its output must match the GPU's
    within the north-star tolerance. Without a snapshot the data are random.
    """

    def __init__(self, cfg: dict, snap: LayerSnapshot | None = None) -> None:
        from oracle import paged_kv_oracle as orc

        self.orc = orc
        self.cfg = cfg
        S, D, Hq, Hkv = cfg["page_size"], cfg["head_dim"], cfg["hq"], cfg["hkv"]
        self.ctx = c3_contexts(cfg) if snap is None else snap.ctx
        npg = (self.ctx + S - 1) // S
        P = int(npg.sum())
        self.tables, cur = [], 0
        if snap is not None:
            for n in npg:
                self.tables.append(list(range(cur, cur + int(n))))
                cur += int(n)
            self.kp = snap.k.permute(0, 1, 3, 2).float().cpu().numpy()
            self.vp = snap.v.permute(0, 1, 3, 2).float().cpu().numpy()
            self.q = snap.q.float().cpu().numpy()
            self.kn = snap.k_new.float().cpu().numpy()
            self.vn = snap.v_new.float().cpu().numpy()
            self.gpu_out = snap.out.float().cpu().numpy()
        else:
            rng = np.random.default_rng(99)
            self.kp = rng.standard_normal((P, Hkv, D, S), dtype=np.float32)
            self.vp = rng.standard_normal((P, Hkv, D, S), dtype=np.float32)
            perm = rng.permutation(P)
            for n in npg:
                self.tables.append([int(x) for x in perm[cur:cur + n]])
                cur += n
            self.q = rng.standard_normal((len(self.ctx), Hq, D), dtype=np.float32)
            self.kn = rng.standard_normal((len(self.ctx), Hkv, D), dtype=np.float32)
            self.vn = self.kn
            self.gpu_out = None
        self.slots = np.array([orc.slot_of(t, int(c) - 1, S) for t, c in zip(self.tables, self.ctx)])
        self.parity = None

    def layer(self) -> np.ndarray:
        self.orc.write_kv_slots(self.kp, self.vp, self.kn, self.vn, self.slots, self.cfg["page_size"])
        return self.orc.paged_attention_decode(self.q, self.kp, self.vp, self.tables, self.ctx,
                                               self.cfg["page_size"])

    def check(self, ref: np.ndarray) -> dict:
        """Compare the GPU's layer-0 output with the oracle's: |gpu - ref| <= 2e-2 + 1e-2 |ref|."""
        err = np.abs(self.gpu_out - ref)
        bad = int((err > 2e-2 + 1e-2 * np.abs(ref)).sum()) + int((~np.isfinite(self.gpu_out)).sum())
        return dict(status="ok" if bad == 0 else "FAIL",
                    checked=f"layer 0 of the timed step: {ref.shape[0]} requests x {ref.shape[1]} "
                            f"query heads x {ref.shape[2]} vs the numpy oracle",
                    tolerance="|out - ref| <= 2e-2 + 1e-2 |ref| (fp32 oracle on the same bf16 inputs)",
                    max_abs_err=float(err.max()), violations=bad)

    def measure(self, target_s: float) -> dict:
        """Run layers until `target_s` seconds of CPU work (at least one); tok/s of a step."""
        cfg = self.cfg
        layers, t0 = 0, time.perf_counter()
        while True:
            out = self.layer()
            if layers == 0 and self.gpu_out is not None:
                self.parity = self.check(out)
            layers += 1
            dt = time.perf_counter() - t0
            if dt >= target_s or layers >= cfg["layers"]:
                break
        scale = cfg["layers"] / layers
        step_s = dt * scale
        return dict(value=round(cfg["batch"] / step_s, 3), unit="tok/s",
                    cores=_blas_threads(), host_cpus=os.cpu_count(), cpu_model=_cpu_model(),
                    kind="port",
                    sample=f"{layers} layer(s) x {len(self.ctx)} requests ({int(self.ctx.sum())} "
                           f"context tokens per layer), fp32 numpy oracle on "
                           f"{'layer 0 of the timed step' if self.gpu_out is not None else 'random data'}"
                           f", scaled x{scale:.2f} to one {cfg['layers']}-layer step; {dt:.1f} s "
                           f"measured")


def _cpu_model() -> str:
    """The host CPU's model name (Linux /proc/cpuinfo), or "unknown"."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:
        pass
    return os.cpu_count() or 1


class ReferenceLayer:
    """One C3 decode layer on the CPU with the reference's own algorithm (its torch
    operations, restated in oracle/ref_torch_path.py): for each of the 64 requests, the
    new K/V row written into a logical [pages, Hkv, D, S] bf16 pool, then gather +
    repeat_interleave + SDPA over its context. bf16 is the pool dtype of the config.
    """

    def __init__(self, cfg: dict) -> None:
        from oracle import ref_torch_path as rtp

        self.rtp = rtp
        self.cfg = cfg
        S, D, Hq, Hkv = cfg["page_size"], cfg["head_dim"], cfg["hq"], cfg["hkv"]
        self.ctx = [int(c) for c in c3_contexts(cfg)]
        npg = [-(-c // S) for c in self.ctx]
        P = sum(npg)
        g = torch.Generator().manual_seed(99)
        self.kp = torch.empty((P, Hkv, D, S), dtype=torch.bfloat16).normal_(generator=g)
        self.vp = torch.empty((P, Hkv, D, S), dtype=torch.bfloat16).normal_(generator=g)
        perm = torch.randperm(P, generator=g).tolist()
        self.tables, cur = [], 0
        for n in npg:
            self.tables.append(perm[cur:cur + n])
            cur += n
        B = len(self.ctx)
        self.q = torch.randn((B, Hq, D), generator=g).to(torch.bfloat16)
        self.kn = torch.randn((B, Hkv, D), generator=g).to(torch.bfloat16)
        self.vn = torch.randn((B, Hkv, D), generator=g).to(torch.bfloat16)

    def run(self) -> None:
        self.rtp.decode_layer(self.q, self.kn, self.vn, self.kp, self.vp, self.tables, self.ctx,
                              self.cfg["page_size"])


def run_reference(args, rank: int, world: int) -> None:
    """The reference's CPU decode KV path, timed on this host's cores (rank 0 only).

    Each timed step is one real layer of the C3 step: all 64 requests' K/V writes and
    attention, as the reference's runner does them (a whole 36-layer step would take
    about a minute per step). `ms_per_step` is that layer's measured time, so `steps` x
    `ms_per_step` is the time actually spent; `value` is the tok/s of the 36-layer step
    those layers add up to (64 tokens per 36 layers).
    """
    if rank != 0:
        return
    cfg = dict(C3)
    torch.set_num_threads(os.cpu_count() or 1)
    layer = ReferenceLayer(cfg)
    for _ in range(args.warmup):
        layer.run()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        layer.run()
        times.append(time.perf_counter() - t0)
    t_layer = sum(times) / len(times)
    v = round(cfg["batch"] / (t_layer * cfg["layers"]), 4)
    sample = (f"one of the step's {cfg['layers']} layers per timed step: 64 requests x (K/V row "
              f"write + gather + repeat_interleave + SDPA), {sum(layer.ctx)} context tokens, bf16 "
              f"pools, torch on {torch.get_num_threads()} threads; tok/s = 64 / (36 x "
              f"{t_layer * 1e3:.1f} ms)")
    cb = dict(value=v, unit="tok/s", cores=torch.get_num_threads(), host_cpus=os.cpu_count(),
              cpu_model=_cpu_model(), kind="port",
              code="the reference's decode path (runner_paged._write_kv_layer + "
                   "attention.paged_attention_v1) restated op for op in oracle/ref_torch_path.py",
              sample=sample)
    line = dict(metric=METRIC, value=v, unit="tok/s", impl="reference", n_gpus=world,
                steps=args.steps, warmup=args.warmup, ms_per_step=round(t_layer * 1e3, 3),
                higher_is_better=True, scaling="strong", vs_baseline=None, dtype="bf16",
                data="synthetic",
                config=dict(workload="C3 qwen3-8b-shape paged decode KV path (36 layers x "
                            "index-copy + paged attention), B=64, ctx U[512,8192]",
                            global_batch=cfg["batch"], layers=cfg["layers"], layers_per_timed_step=1,
                            parallelism="cpu reference (torch ops of the reference path)"),
                cpu_baseline=cb,
                e2e=dict(value=v, unit="tok/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), flush=True)


def run_c2_only(args, dev: torch.device) -> None:
    """C2 index-copy microbench alone (with --profile: plain launches for ncu)."""
    from plastic_infer_b200 import kernels

    peaks = measured_peaks()
    if not args.profile:
        print(json.dumps(dict(index_copy=bench_index_copy(dev, peaks["hbm_gbs"]))), flush=True)
        return
    P, S, H, D = C2["pages"], C2["page_size"], C2["hkv"], C2["head_dim"]
    kp = torch.zeros((P, H, S, D), dtype=torch.bfloat16, device=dev)
    vp = torch.zeros_like(kp)
    perm = np.random.default_rng(0).permutation(P * S)
    for B in C2["batches"]:
        slots = torch.from_numpy(perm[:B].astype(np.int64)).to(dev)
        kn = torch.randn((B, H, D), dtype=torch.bfloat16, device=dev)
        vn = torch.randn((B, H, D), dtype=torch.bfloat16, device=dev)
        for _ in range(args.warmup + args.steps):
            kernels.kv_index_copy(kp, vp, kn, vn, slots)
    torch.cuda.synchronize()
    print(json.dumps(dict(profile=True, c2_batches=list(C2["batches"]))), flush=True)


def c5_prefill(cfg: dict, dev: torch.device, hkv: int):
    """C5 state of one rank through the host KV store API: B requests of `ctx` tokens and
    this rank's `hkv` KV heads, written chunk by chunk into a device pool that holds
    `pool_frac` of all pages; every chunk is sunk to the pinned host store as it completes,
    and the oldest sunk chunks are evicted to make room for the next one. Returns
    (store, caches, decoder)."""
    from plastic_infer_b200 import kernels
    from plastic_infer_b200.decode import HostStoreDecoder
    from plastic_infer_b200.kv.kv_store import KVConfig, KVStore

    L, B, S, D = (cfg[x] for x in ("layers", "batch", "page_size", "head_dim"))
    ppc = cfg["pages_per_chunk"]
    tpc = S * ppc
    total_pages = L * B * cfg["ctx"] // S
    pool = int(cfg["pool_frac"] * total_pages)
    kvc = KVConfig(n_layers=L, n_kv_heads=hkv, head_dim=D, page_size=S, pages_per_chunk=ppc,
                   max_pages=pool, max_host_chunks=B * (cfg["ctx"] // tpc) + B,
                   dtype=torch.bfloat16, device=dev)
    store = KVStore(kvc)
    caches = [store.new_request(request_id=b) for b in range(B)]
    # headroom for one decode step's new pages (a page per layer per request)
    dec = HostStoreDecoder(store, caches, budget_pages=pool - L * B)
    g = torch.Generator(device=dev).manual_seed(cfg["seed"])
    rows_k = torch.empty((L * tpc, hkv, D), dtype=torch.bfloat16, device=dev)
    rows_v = torch.empty_like(rows_k)
    rng = np.random.default_rng(cfg["seed"])
    chunk_pages = L * ppc
    offs = np.arange(tpc, dtype=np.int64)
    for c in range(cfg["ctx"] // tpc):
        for cache in caches:
            dec.evict_to(pool - chunk_pages)  # room for this chunk
            start = cache.length
            cache.reserve_tokens(tpc)
            # slots of the chunk's tokens in every layer (layer-major rows)
            pos = start + offs
            slots = np.concatenate([np.asarray(cache.block_table.pages[l], dtype=np.int64)[pos // S] * S
                                    + pos % S for l in range(L)])
            rows_k.normal_(generator=g)
            rows_v.normal_(generator=g)
            kernels.kv_index_copy(store.gpu.k_phys, store.gpu.v_phys, rows_k, rows_v,
                                  torch.from_numpy(slots).to(dev))
            cache.extend_token_ids([int(x) for x in rng.integers(0, 151936, tpc)])
            store.sink_completed_chunks_async(cache)
    dec.evict_to(dec.budget)
    torch.cuda.synchronize()
    return store, caches, dec


def host_link_gbs(dev: torch.device) -> float:
    """Pinned 1 GiB host->device copy rate of this GPU's link (GB/s)."""
    h = torch.empty(1 << 30, dtype=torch.uint8, pin_memory=True)
    d = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
    d.copy_(h)
    torch.cuda.synchronize()
    ms = time_region(lambda: d.copy_(h, non_blocking=True), 3, torch.cuda.current_stream()) / 3
    del h, d
    return (1 << 30) / (ms * 1e-3) / 1e9


def c5_parity(store, caches, q: torch.Tensor, out: torch.Tensor, checks) -> dict:
    """Outputs of the last C5 step against the oracle, for (request, layer) pairs `checks`:
    each request's whole K/V history of that layer is rebuilt independently of the decode
    path, from its evicted chunks in the host store and its device pages, and the oracle
    attends this rank's query heads over it."""
    from oracle import paged_kv_oracle as orc

    cfg = store.config
    S, ppc, tpc = cfg.page_size, cfg.pages_per_chunk, cfg.tokens_per_chunk
    worst, bad, tokens = 0.0, 0, 0
    for b, layer in checks:
        c = caches[b]
        T = c.length
        ks, vs = [], []
        for ci in range(c.evicted_chunks):  # host chunks: logical [L, H, D, tpc]
            hk, hv = store._host_cache[c.chunk_keys[ci].full_key]
            ks.append(hk[layer].float().permute(2, 0, 1))
            vs.append(hv[layer].float().permute(2, 0, 1))
        pages = c.block_table.pages[layer][c.evicted_chunks * ppc:-(-T // S)]
        idx = torch.tensor(pages, dtype=torch.int64, device=store.gpu.k_phys.device)
        for pool, dst in ((store.gpu.k_phys, ks), (store.gpu.v_phys, vs)):  # [P, H, S, D]
            rows = pool.index_select(0, idx).permute(0, 2, 1, 3).reshape(-1, pool.shape[1], pool.shape[3])
            dst.append(rows[:T - c.evicted_chunks * tpc].float().cpu())
        k = torch.cat(ks).numpy()
        v = torch.cat(vs).numpy()
        npg = -(-T // S)
        pad = np.zeros((npg * S - T,) + k.shape[1:], np.float32)
        kp = np.concatenate([k, pad]).reshape(npg, S, k.shape[1], k.shape[2]).transpose(0, 2, 3, 1)
        vp = np.concatenate([v, pad]).reshape(npg, S, v.shape[1], v.shape[2]).transpose(0, 2, 3, 1)
        ref = orc.paged_attention_decode(q[layer, b].float().cpu().numpy()[None], kp, vp,
                                         [list(range(npg))], [T], S)[0]
        got = out[layer, b].float().cpu().numpy()
        err = np.abs(got - ref)
        worst = max(worst, float(err.max()))
        bad += int((err > 2e-2 + 1e-2 * np.abs(ref)).sum()) + int((~np.isfinite(got)).sum())
        tokens += T
    return dict(status="ok" if bad == 0 else "FAIL",
                checked=f"last timed step, (request, layer) {list(checks)}: each history "
                        f"({tokens} tokens in all) rebuilt from the host chunks and device pages, "
                        "this rank's query heads vs the numpy oracle",
                tolerance="|out - ref| <= 2e-2 + 1e-2 |ref| (fp32 oracle on the same bf16 inputs)",
                max_abs_err=worst, violations=bad)


def measure_c5(args, rank: int, world: int, dev: torch.device, steps: int, warmup: int) -> dict:
    """C5 long-context decode through the KV store API on every rank of the job.

    KV heads are split over the ranks (rank r keeps heads [r*8/N, (r+1)*8/N) of every
    request, its share of the pool, and its own pinned host store), so each rank streams its
    own host chunks over its own host link; per layer the ranks' attention outputs are
    all-gathered (NCCL) before o_proj would run. Each step runs HostStoreDecoder: per layer
    the new K/V rows are written and every request is attended by host-stream attention over
    its evicted chunks (read in place) plus its device tail; completed chunks are sunk on
    the store's side stream and evicted to the pool budget. The roofline is the host link:
    host bytes read per step over the step time, against the pinned copy rate the ranks
    reach together (each copying 1 GiB at the same time). A rank that fails to build its
    state makes every rank skip the timed part (no collective is left waiting).
    """
    import torch.distributed as dist

    from plastic_infer_b200.dist import head_shard

    cfg = dict(C5)
    if args.layers:
        cfg["layers"] = args.layers
    L, B, D, Hkv, Hq = (cfg[x] for x in ("layers", "batch", "head_dim", "hkv", "hq"))
    tpc = cfg["page_size"] * cfg["pages_per_chunk"]
    err = ""
    try:
        shard = head_shard(Hq, Hkv, world, rank)
        t0 = time.perf_counter()
        store, caches, dec = c5_prefill(cfg, dev, shard.n_kv)
        prefill_s = time.perf_counter() - t0
    except Exception as e:  # noqa: BLE001 - reported in the line, every rank skips
        err = f"{type(e).__name__}: {e}"[:200]
    ok = torch.tensor([0.0 if err else 1.0], device=dev)
    if world > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if ok.item() < 1.0:
        return dict(skipped=err or "another rank could not build its C5 state")
    # every rank copies at the same time: the host side of the links is shared, so the
    # peak is what the ranks reach together, not one link alone
    barrier(world)
    link = host_link_gbs(dev)
    g = torch.Generator(device=dev).manual_seed(cfg["seed"] + 1)
    q = torch.randn((L, B, shard.n_q, D), dtype=torch.bfloat16, device=dev, generator=g)
    kn = torch.randn((L, B, shard.n_kv, D), dtype=torch.bfloat16, device=dev, generator=g)
    vn = torch.randn((L, B, shard.n_kv, D), dtype=torch.bfloat16, device=dev, generator=g)
    out = torch.empty_like(q)
    gathered = (torch.empty((L, world * B, shard.n_q, D), dtype=torch.bfloat16, device=dev)
                if world > 1 else None)
    rng = np.random.default_rng(cfg["seed"] + 2)
    chunk_layer_bytes = 2 * tpc * shard.n_kv * D * 2    # K + V of one chunk of one layer

    def step():
        ids = [int(x) for x in rng.integers(0, 151936, B)]
        dec.begin_step(ids)
        for layer in range(L):
            dec.attend(layer, q[layer], kn[layer], vn[layer], out=out[layer])
            if gathered is not None:
                dist.all_gather_into_tensor(gathered[layer], out[layer])
        dec.end_step()

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    host_bytes = 0
    barrier(world)
    with ClockSampler(list(range(world)) if rank == 0 else None) as clk:
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        if world > 1:
            dist.all_reduce(torch.zeros(1, device=dev))
        start.record()
        for _ in range(steps):
            host_bytes += sum(c.evicted_chunks for c in caches) * chunk_layer_bytes * L
            step()
        end.record()
        torch.cuda.synchronize()
        ms = start.elapsed_time(end)
    barrier(world)
    ms = max_over_ranks(ms, world)
    totals = torch.tensor([float(host_bytes), link], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(totals)
    hb, link_sum = float(totals[0]) / steps, float(totals[1])
    ms_step = ms / steps
    res = dict(
        metric="decode tok/s (long-context host offload, Qwen3-8B attention shape)",
        value=round(B * steps / (ms * 1e-3), 2), unit="tok/s", n_gpus=world, steps=steps,
        warmup=warmup, ms_per_step=round(ms_step, 2),
        workload=f"C5 through the KV store API: B={B} x {cfg['ctx']} tokens, {L} layers, "
                 f"{Hq}q/{Hkv}kv heads (kv-head shard x{world}), head_dim {D}; device pool = "
                 f"{cfg['pool_frac']:.0%} of all pages; per layer index-copy + host-stream "
                 "attention over the evicted chunks (pinned, read in place) and the device "
                 "tail; async sink + eviction to the pool budget after every step",
        evicted_chunks_per_rank=sum(c.evicted_chunks for c in caches),
        prefill_s=round(prefill_s, 1),
        roofline=dict(bound="host link", achieved=round(hb / (ms_step * 1e-3) / 1e9, 1),
                      peak=round(link_sum, 1), unit="GB/s",
                      frac=round(hb / (ms_step * 1e-3) / 1e9 / link_sum, 3),
                      peak_source="sum over the ranks of a pinned 1 GiB host->device copy, all "
                                  "ranks copying at once, measured in this run"),
        host_bytes_read_per_step=int(hb), clocks=clk.summary())
    if rank == 0 and not args.skip_cpu:
        res["parity"] = c5_parity(store, caches, q, out, [(0, 0), (B - 1, L - 1)])
    del store, caches, dec, q, kn, vn, out, gathered
    torch.cuda.empty_cache()
    return res


def run_c5(args, rank: int, world: int, dev: torch.device) -> None:
    """C5 long-context offload line (`--workload c5`), on every rank of the job."""
    res = measure_c5(args, rank, world, dev, args.steps, args.warmup)
    if rank == 0:
        line = dict(res)
        workload = line.pop("workload", "C5")
        line.update(scaling="strong", higher_is_better=True, vs_baseline=None, dtype="bf16",
                    data="synthetic", config=dict(workload=workload))
        print(json.dumps(line), flush=True)
        if res.get("parity", {}).get("status", "ok") != "ok":
            raise SystemExit("parity check of the C5 step failed: " + json.dumps(res["parity"]))


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if args.c2_only:
        run_c2_only(args, dev)
        return
    if args.host_stream_only:
        print(json.dumps(dict(host_stream=bench_host_stream(dev))), flush=True)
        return
    if args.prefill_only:
        print(json.dumps(dict(prefill=bench_prefill(dev, measured_peaks()))), flush=True)
        return
    if args.page_copy_only:
        print(json.dumps(dict(page_copy=bench_page_copy(dev, measured_peaks()["hbm_gbs"],
                                                        profile=args.profile))), flush=True)
        return
    if args.expert_copy_only:
        print(json.dumps(dict(expert_copy=bench_expert_copy(dev))), flush=True)
        return
    if args.prologue_only:
        print(json.dumps(dict(decode_prologue=bench_prologue(dev, measured_peaks()["hbm_gbs"]))),
              flush=True)
        return
    if args.workload == "c5":
        run_c5(args, rank, world, dev)
        return
    peaks = measured_peaks()
    cfg = dict(WORKLOADS[args.workload])
    if args.layers:
        cfg["layers"] = args.layers
    # Programmatic dependent launch: each attention computes its work split and fetches
    # its first page ids while the step's index-copy runs, then waits for it; every
    # kernel still reads its inputs only after the kernel before it has completed.
    from plastic_infer_b200 import kernels

    kernels.set_programmatic_launch(not args.no_pdl)
    kernels.set_decode_attn_ring(args.attn_ring)
    wl = DecodeWorkload(cfg, rank, world, dev)
    wl.fused = args.fused
    if world > 1 and not args.nccl:
        wl.use_peer_gather()
    stream = torch.cuda.current_stream()

    # warm-up (also configures kernels before graph capture)
    for _ in range(max(1, args.warmup)):
        wl.step()
    torch.cuda.synchronize()
    if args.profile:
        # Profiling mode (ncu): plain launches, nothing but the timed steps.
        for _ in range(args.steps):
            wl.step()
        torch.cuda.synchronize()
        if rank == 0:
            print(json.dumps(dict(profile=True, layers=cfg["layers"], steps=args.steps,
                                  attn_bytes_per_launch=int(wl.attn_bytes()))), flush=True)
        return
    # The whole step is one CUDA graph at N = 1 and with the fused peer all-gather at
    # N > 1 (its launches take their epochs from a device counter, so one capture
    # replays every step). With --nccl the step runs eagerly: a captured NCCL
    # all-gather of the 512 KB per-layer output measured ~25 us per layer on B200 x2,
    # slower than the eager launch sequence. Graphs are dropped before the process
    # group is destroyed.
    use_graph = not args.no_graph and (world == 1 or wl.exchange is not None)
    step_fn = wl.step
    if use_graph:
        g_step = graph_of(wl.step)
        step_fn = g_step.replay
        for _ in range(args.warmup):
            step_fn()

    barrier(world)
    with ClockSampler(list(range(world)) if rank == 0 else None) as clk:
        ms = time_region(step_fn, args.steps, stream, world)
    barrier(world)
    ms = max_over_ranks(ms, world)
    ms_step = ms / args.steps
    value = cfg["batch"] * args.steps / (ms * 1e-3)
    # Layer 0 of the step just timed, for the CPU baseline leg's parity check (N = 1).
    check_cpu = rank == 0 and world == 1 and not args.skip_cpu
    snap = LayerSnapshot(wl) if check_cpu else None

    # attention alone (dominant kernel), same stream, for the roofline
    attn_fn = lambda: wl.step(attention=True, copy=False, gather=False)  # noqa: E731
    copy_fn = lambda: wl.step(attention=False, copy=True, gather=False)  # noqa: E731
    if use_graph:
        ga, gc = graph_of(attn_fn), graph_of(copy_fn)
        attn_fn, copy_fn = ga.replay, gc.replay
    reps = max(2, args.steps)
    attn_ms = time_region(attn_fn, reps, stream, world) / (reps * cfg["layers"])
    copy_ms = time_region(copy_fn, reps, stream, world) / (reps * cfg["layers"])
    attn_ms = max_over_ranks(attn_ms, world)
    achieved = wl.attn_bytes() / (attn_ms * 1e-3) / 1e9

    # e2e through the public API with pinned host buffers
    e2e = None
    if not args.skip_e2e:
        e2e = run_e2e(wl, args, stream, use_graph)
    # the C4 and C5 shapes on the same ranks (every N of a scaling run records them); C5
    # with a few steps (one takes ~0.6 s on one GPU)
    c4 = (measure_c4(args, rank, world, dev, peaks)
          if args.workload == "c3" and not args.skip_c4 else None)
    c5 = (measure_c5(args, rank, world, dev, steps=min(args.steps, 5), warmup=2)
          if args.workload == "c3" and not args.skip_c5 else None)

    idx = (bench_index_copy(dev, peaks["hbm_gbs"])
           if (world == 1 and not args.skip_c2 and args.workload == "c3") else None)
    pro = (bench_prologue(dev, peaks["hbm_gbs"])
           if (world == 1 and not args.skip_c2 and args.workload == "c3") else None)
    cpu, parity = None, None
    if check_cpu:
        sample = CpuSample(cfg, snap)
        del snap
        cpu = sample.measure(12.0)
        parity = sample.parity
        del sample

    # measured DRAM bytes per launch exist for the C3 single-GPU launch only
    traffic = _profile_traffic() if (args.workload == "c3" and world == 1) else None
    if rank == 0:
        line = dict(
            metric=cfg.get("metric", METRIC), value=round(value, 1), unit="tok/s", n_gpus=world,
            steps=args.steps,
            warmup=args.warmup, ms_per_step=round(ms_step, 4), higher_is_better=True,
            scaling="strong", vs_baseline=None, dtype="bf16", data="synthetic",
            config=dict(workload=cfg["desc"] + ("" if cfg["layers"] == WORKLOADS[args.workload]["layers"]
                                                 else f" (profiling run: {cfg['layers']} layers)"),
                        global_batch=cfg["batch"], layers=cfg["layers"],
                        seq_len=f"ragged {cfg['ctx_lo']}-{cfg['ctx_hi']}",
                        parallelism=(f"kv-head shard x{world}, "
                                     + ("NCCL all-gather" if args.nccl else
                                        "all-gather fused into the attention kernel (NVLink peer stores)")
                                     if world > 1 else "single gpu"),
                        kv_bytes_per_step=round(wl.attn_bytes() * cfg["layers"] * world / 1e9, 3),
                        l2=f"inputs larger than L2 "
                           f"(~{wl.attn_bytes() * cfg['layers'] / 1e9:.0f} GB KV per step), no flush",
                        cuda_graph=use_graph, programmatic_launch=not args.no_pdl,
                        attn_ring=args.attn_ring),
            roofline=dict(bound="hbm", achieved=round(achieved, 1), peak=peaks["hbm_gbs"],
                          unit="GB/s", frac=round(achieved / peaks["hbm_gbs"], 4),
                          traffic=traffic, kernel="paged_decode_attn_tma_kernel<bf16,128,16>",
                          us_per_launch=round(attn_ms * 1e3, 2),
                          algorithmic_bytes_per_launch=int(wl.attn_bytes()),
                          peak_source=peaks["source"]),
            index_copy_in_step=dict(us_per_launch=round(copy_ms * 1e3, 2),
                                    gbs=round(wl.copy_bytes() / (copy_ms * 1e-3) / 1e9, 1)),
            gpu_launches=args.steps * cfg["layers"] * (1 if wl.fused else 2),
            clocks=clk.summary(),
        )
        if e2e is not None:
            line["e2e"] = e2e
        if idx is not None:
            line["index_copy"] = dict(workload="C2: 65536-page bf16 pool x 16 x 8 x 128, "
                                      "random distinct slots", bytes_per_row=8200,
                                      per_batch=idx, peak=peaks["hbm_gbs"])
        if pro is not None:
            line["decode_prologue"] = dict(
                workload="fused QK-norm + RoPE + K/V slot write of one decode layer (bf16, D=128, "
                         "theta 1e6, positions < 8192) vs the reference's unfused GPU ops",
                per_shape=pro, peak=peaks["hbm_gbs"])
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if c4 is not None:
            line["c4"] = c4
        if c5 is not None:
            line["c5"] = c5
        line["parity"] = parity if parity is not None else dict(
            status="not checked in this run",
            why=("the check runs in the N=1 CPU baseline leg; the sharded path is checked by "
                 "tests/test_gpu_multi.py") if world > 1 else "--skip-cpu")
        print(json.dumps(line), flush=True)
    # release graphs (they may hold NCCL work) before the process group goes away
    step_fn = attn_fn = copy_fn = None
    if use_graph:
        del g_step, ga, gc
    torch.cuda.synchronize()
    barrier(world)
    if wl.exchange is not None:
        wl.exchange.close()
        barrier(world)
    if parity is not None and parity["status"] != "ok":
        raise SystemExit("parity check of the timed step failed: " + json.dumps(parity))
    for name, leg in (("C4", c4), ("C5", c5)):
        if leg is not None and leg.get("parity", {}).get("status", "ok") != "ok":
            raise SystemExit(f"parity check of the {name} step failed: " + json.dumps(leg["parity"]))


def measure_c4(args, rank: int, world: int, dev: torch.device, peaks: dict) -> dict:
    """The C4 (Qwen3-30B-A3B shape) KV path on the same ranks as the C3 line: the same
    sharding (a KV head per rank is replicated when there are fewer KV heads than ranks),
    gather and graph capture; device time is the max over ranks. At N = 1 (unless
    --skip-cpu) layer 0 of the timed step is checked against the oracle, like the C3 line."""
    from plastic_infer_b200 import kernels

    cfg = dict(C4)
    wl = DecodeWorkload(cfg, rank, world, dev)
    if world > 1 and not args.nccl:
        wl.use_peer_gather()
    stream = torch.cuda.current_stream()
    for _ in range(max(1, args.warmup)):
        wl.step()
    torch.cuda.synchronize()
    use_graph = not args.no_graph and (world == 1 or wl.exchange is not None)
    step_fn, g_step, g_attn = wl.step, None, None
    if use_graph:
        g_step = graph_of(wl.step)
        step_fn = g_step.replay
        for _ in range(args.warmup):
            step_fn()
    barrier(world)
    ms = max_over_ranks(time_region(step_fn, args.steps, stream, world), world)
    attn_fn = lambda: wl.step(attention=True, copy=False, gather=False)  # noqa: E731
    if use_graph:
        g_attn = graph_of(attn_fn)
        attn_fn = g_attn.replay
    reps = max(2, args.steps)
    attn_ms = max_over_ranks(time_region(attn_fn, reps, stream, world) / (reps * cfg["layers"]),
                             world)
    achieved = wl.attn_bytes() / (attn_ms * 1e-3) / 1e9
    D, S = cfg["head_dim"], cfg["page_size"]
    ring = kernels.decode_attn_ring_stages(cfg["batch"], wl.block_tables.shape[2], wl.hq, wl.hkv,
                                           D, S, wl.k_pool.shape[0], torch.bfloat16)
    res = dict(workload=cfg["desc"], metric=cfg["metric"],
               value=round(cfg["batch"] * args.steps / (ms * 1e-3), 1), unit="tok/s",
               n_gpus=world, ms_per_step=round(ms / args.steps, 4),
               parallelism=(f"kv-head shard x{world}" + (" (KV heads replicated)"
                                                         if world > cfg["hkv"] else "")
                            if world > 1 else "single gpu"),
               roofline=dict(bound="hbm", kernel="paged_decode_attn_tma_kernel<bf16,128,16>",
                             ring_stages=ring, us_per_launch=round(attn_ms * 1e3, 2),
                             algorithmic_bytes_per_launch=int(wl.attn_bytes()),
                             achieved=round(achieved, 1), peak=peaks["hbm_gbs"], unit="GB/s",
                             frac=round(achieved / peaks["hbm_gbs"], 4)))
    if world == 1 and not args.skip_cpu:
        sample = CpuSample(cfg, LayerSnapshot(wl))
        res["parity"] = sample.check(sample.layer())
        del sample
    step_fn = attn_fn = None
    del g_step, g_attn
    torch.cuda.synchronize()
    barrier(world)
    if wl.exchange is not None:
        wl.exchange.close()
        barrier(world)
    del wl
    torch.cuda.empty_cache()
    return res


def run_e2e(wl: DecodeWorkload, args, stream, use_graph: bool = False) -> dict:
    """Whole step through the public API, inputs from pinned host memory each step.

    Layer l's inputs are copied host->device on one copy stream and its attention
    output device->host on another, so the copies of layer l+1 / l-1 overlap the
    kernels of layer l; the step ends when the last output is on the host. With
    `use_graph` the step (copies, kernels and the streams' event edges) is captured once
    through the same API calls and replayed: every replay copies that step's inputs in
    and its outputs out.
    """
    from plastic_infer_b200 import kernels

    # Each rank feeds its own shard (its KV heads' new rows and its query heads) from
    # its own pinned buffers; with N > 1 the per-layer outputs are all-gathered and
    # rank 0 reads the gathered [B, Hq, D] result back.
    q_h = wl.q.cpu().pin_memory()
    kn_h = wl.k_new.cpu().pin_memory()
    vn_h = wl.v_new.cpu().pin_memory()
    L = wl.cfg["layers"]
    result = wl.gathered if wl.world > 1 else wl.out
    out_h = torch.empty(result.shape, dtype=result.dtype, pin_memory=True)
    if wl.exchange is not None:
        # one slot per layer: layer l's gathered output is slot l of this rank's buffer
        result = [wl.exchange.slot_tensor(s) for s in range(L)]
    read_back = wl.world == 1 or int(os.environ.get("RANK", "0")) == 0
    q_d, kn_d, vn_d = torch.empty_like(wl.q), torch.empty_like(wl.k_new), torch.empty_like(wl.v_new)
    slots_d = torch.empty_like(wl.slots)
    ctx_d = torch.empty_like(wl.ctx_lens)
    L = wl.cfg["layers"]
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(L)]
    ev_out = [torch.cuda.Event() for _ in range(L)]
    ev_read = [torch.cuda.Event() for _ in range(L)]

    def step():
        cur = torch.cuda.current_stream()  # the capture stream while capturing
        h2d.wait_stream(cur)  # device inputs of the previous step are no longer read
        with torch.cuda.stream(h2d):
            ctx_d.copy_(wl.ctx_host, non_blocking=True)
            for l in range(L):
                q_d[l].copy_(q_h[l], non_blocking=True)
                kn_d[l].copy_(kn_h[l], non_blocking=True)
                vn_d[l].copy_(vn_h[l], non_blocking=True)
                slots_d[l].copy_(wl.slots_host[l], non_blocking=True)
                ev_in[l].record(h2d)
        for l in range(L):
            cur.wait_event(ev_in[l])
            if wl.exchange is not None and read_back and l >= 2:
                # Peers store into this rank's slots without waiting for its reads: a
                # peer's launch e starts once this rank has finished launch e - 1, so
                # the read of a slot's previous output must be done before this rank's
                # launch e - 1 starts. Waiting here for the read issued two launches back
                # keeps that within the step and still lets each read overlap the next
                # launch; across steps the end-of-step wait on the copy stream keeps it.
                cur.wait_event(ev_read[l - 2])
            if wl.exchange is not None:
                kernels.kv_index_copy(wl.k_pool, wl.v_pool, kn_d[l], vn_d[l], slots_d[l])
                kernels.paged_decode_attention_gather(q_d[l], wl.k_pool, wl.v_pool,
                                                      wl.block_tables[l], ctx_d, wl.exchange,
                                                      workspace=wl.ws)
            elif wl.fused:
                kernels.paged_decode_attention(q_d[l], wl.k_pool, wl.v_pool, wl.block_tables[l],
                                               ctx_d, out=wl.out[l], workspace=wl.ws,
                                               k_new=kn_d[l], v_new=vn_d[l], slot_mapping=slots_d[l])
            else:
                kernels.kv_index_copy(wl.k_pool, wl.v_pool, kn_d[l], vn_d[l], slots_d[l])
                kernels.paged_decode_attention(q_d[l], wl.k_pool, wl.v_pool, wl.block_tables[l],
                                               ctx_d, out=wl.out[l], workspace=wl.ws)
            if wl.world > 1 and wl.exchange is None:
                import torch.distributed as dist

                dist.all_gather_into_tensor(wl.gathered[l], wl.out[l])
            ev_out[l].record(cur)
            if read_back:
                # a gather launch ends once every rank's slice is here: read it now
                with torch.cuda.stream(d2h):
                    d2h.wait_event(ev_out[l])
                    out_h[l].copy_(result[l], non_blocking=True)
                    ev_read[l].record(d2h)
        if read_back:
            cur.wait_stream(d2h)

    for _ in range(args.warmup):
        step()
    step_fn = step
    if use_graph:
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        step_fn = graph.replay
        for _ in range(args.warmup):
            step_fn()
    barrier(wl.world)
    ms = max_over_ranks(time_region(step_fn, args.steps, stream, wl.world), wl.world)
    # whole job: every rank copies its shard in; rank 0 reads the result out
    h2d = wl.world * sum(t.numel() * t.element_size()
                         for t in (q_h, kn_h, vn_h, wl.slots_host, wl.ctx_host))
    d2h = out_h.numel() * out_h.element_size()
    return dict(value=round(wl.cfg["batch"] * args.steps / (ms * 1e-3), 1), unit="tok/s",
                h2d_bytes_per_step=int(h2d), d2h_bytes_per_step=int(d2h),
                ms_per_step=round(ms / args.steps, 4), api="plastic_infer_b200.kernels",
                cuda_graph=use_graph)


def _profile_traffic():
    """DRAM bytes per attention launch from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        try:
            with open(path) as f:
                return json.load(f).get("paged_decode_attn_c3_bytes_per_launch")
        except (OSError, ValueError):
            return None
    return None


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-c2", action="store_true", help="skip the index-copy microbench")
    ap.add_argument("--skip-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--skip-e2e", action="store_true", help="skip the host-buffer e2e run")
    ap.add_argument("--skip-c4", action="store_true",
                    help="skip the C4 (Qwen3-30B-A3B shape) line inside the C3 run")
    ap.add_argument("--skip-c5", action="store_true",
                    help="skip the C5 (long context through the host store) line inside the C3 run")
    ap.add_argument("--layers", type=int, default=0,
                    help="decoder layers per step (default: the workload's; fewer only for profiling)")
    ap.add_argument("--workload", choices=["c3", "c4", "c5"], default="c3",
                    help="c3: Qwen3-8B shape (headline); c4: Qwen3-30B-A3B shape; "
                         "c5: long-context host offload")
    ap.add_argument("--profile", action="store_true",
                    help="ncu mode: warm-up + timed steps as plain launches, no extra parts")
    ap.add_argument("--c2-only", action="store_true", help="run only the C2 index-copy microbench")
    ap.add_argument("--host-stream-only", action="store_true",
                    help="print only the host-stream attention microbench (C5 shape)")
    ap.add_argument("--prefill-only", action="store_true",
                    help="run only the paged prefill attention microbench")
    ap.add_argument("--page-copy-only", action="store_true",
                    help="run only the page gather/scatter microbench (with --profile: plain "
                         "launches for ncu)")
    ap.add_argument("--expert-copy-only", action="store_true",
                    help="run only the MoE expert-slot copy microbench")
    ap.add_argument("--prologue-only", action="store_true",
                    help="run only the fused decode-prologue microbench")
    ap.add_argument("--no-graph", action="store_true", help="launch every kernel from Python")
    ap.add_argument("--nccl", action="store_true",
                    help="N > 1: gather the per-layer outputs with NCCL all-gather instead of the "
                         "kernel's NVLink peer stores")
    ap.add_argument("--no-pdl", action="store_true",
                    help="launch kernels without programmatic dependent launch (each attention "
                         "then computes its work split only after the previous kernel ends)")
    ap.add_argument("--attn-ring", choices=["auto", "deep", "shallow"], default="auto",
                    help="page-ring depth of the decode attention (default: chosen per launch)")
    ap.add_argument("--fused", action="store_true",
                    help="one fused append+attention launch per layer instead of index-copy "
                         "then attention (measured slower: 202.9 vs 197.5 us per layer, 4-stage ring)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
