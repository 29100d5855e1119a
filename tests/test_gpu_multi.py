"""Multi-GPU KV-head sharding on real GPUs (row e): NCCL and the fused peer all-gather.

Each rank (one process per GPU, NCCL) holds only its KV heads' pools, attends its
query heads with the sm_100a kernel, and the outputs are gathered:
  * through pi_paged_decode_attn_gather: the kernel pushes its finished row groups to
    every peer's gathered buffer with NVLink stores and ends once every rank's slice
    has landed, so the buffer is read in stream order right after the launch;
  * through dist.gather_heads (NCCL all-gather) as the reference point.
Both must equal, bit for bit, every shard attended on one GPU by the same kernel and
concatenated, and agree with the unsharded kernel within the attention tolerance, for
consecutive launches (slots and epochs rotate), with epochs from the host and from the
device counter, for a CUDA graph of launches replayed with new inputs, for a KV head
replicated on every rank (fewer KV heads than ranks), and with programmatic launch on. Skipped unless at least two
GPUs are visible.
"""

from __future__ import annotations

import os
import socket
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu

NGPU = torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import datetime

    import torch.distributed as dist

    from plastic_infer_b200 import kernels
    from plastic_infer_b200.dist import PeerExchange, gather_heads, head_shard

    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        B, Hq, Hkv, D, S = 12, 32, 8, 128, 16
        g = torch.Generator().manual_seed(0)
        ctx = torch.randint(1, 900, (B,), generator=g)
        ctx[0] = 0  # an empty request is gathered as zeros too
        npg = (ctx + S - 1) // S
        P = int(npg.sum()) + 4
        perm = torch.randperm(P, generator=g)
        bt = torch.zeros((B, int(npg.max())), dtype=torch.int32)
        cur = 0
        for b in range(B):
            bt[b, :npg[b]] = perm[cur:cur + npg[b]].to(torch.int32)
            cur += int(npg[b])
        shard = head_shard(Hq, Hkv, world, rank)
        bt_d = bt.to(dev)
        ctx_d = ctx.to(torch.int32).to(dev)
        ws = kernels.Workspace(dev)

        def inputs(hq=Hq, hkv=Hkv):
            sh = head_shard(hq, hkv, world, rank)
            q = torch.randn((B, hq, D), generator=g).to(torch.bfloat16).to(dev)
            kp = torch.randn((P, hkv, S, D), generator=g).to(torch.bfloat16).to(dev)
            vp = torch.randn((P, hkv, S, D), generator=g).to(torch.bfloat16).to(dev)
            return (q, kp, vp, q[:, sh.q_lo:sh.q_hi].contiguous(),
                    kp[:, sh.kv_lo:sh.kv_hi].contiguous(),
                    vp[:, sh.kv_lo:sh.kv_hi].contiguous())

        def expected(q, kp, vp):
            # bit-exact reference: every shard attended on this GPU with the same kernel
            # (same work split as on its owner rank), concatenated in rank order
            parts = []
            for r in range(world):
                sr = head_shard(q.shape[1], kp.shape[1], world, r)
                parts.append(kernels.paged_decode_attention(
                    q[:, sr.q_lo:sr.q_hi].contiguous(), kp[:, sr.kv_lo:sr.kv_hi].contiguous(),
                    vp[:, sr.kv_lo:sr.kv_hi].contiguous(), bt_d, ctx_d))
            return torch.cat(parts, dim=1)

        def as_heads(gathered, hq=Hq):
            nq = hq // world
            return gathered.view(world, B, nq, D).permute(1, 0, 2, 3).reshape(B, hq, D)

        ok, msg = True, ""

        def check(tag, got, q, kp, vp, nccl=None):
            nonlocal ok, msg
            expect = expected(q, kp, vp)
            full = kernels.paged_decode_attention(q, kp, vp, bt_d, ctx_d)
            close = (got.float() - full.float()).abs().max().item()
            good = torch.equal(got, expect) and close < 2e-2
            if nccl is not None:
                good = good and torch.equal(nccl, expect)
            if not good and ok:
                ok = False
                msg = (f"{tag}: fused==local {torch.equal(got, expect)} max|fused-full| "
                       f"{close:.3e} max|fused-local| "
                       f"{(got.float() - expect.float()).abs().max().item():.3e}")

        # 1) device epochs, eager, consecutive launches (slots and epochs rotate). The
        #    gathered buffer is read in stream order right after the launch: no
        #    synchronize or barrier, the launch itself ends once every slice is here.
        ex = PeerExchange(B, shard.n_q, D, torch.bfloat16)
        for step in range(3):
            q, kp, vp, ql, kpl, vpl = inputs()
            snap = as_heads(kernels.paged_decode_attention_gather(
                ql, kpl, vpl, bt_d, ctx_d, ex, workspace=ws)).clone()
            via_nccl = gather_heads(kernels.paged_decode_attention(ql, kpl, vpl, bt_d, ctx_d), shard)
            check(f"device-epoch step {step}", snap, q, kp, vp, via_nccl)

        # 2) host epochs (launch_counter NULL): the same results
        exh = PeerExchange(B, shard.n_q, D, torch.bfloat16, device_epochs=False)
        for step in range(2):
            q, kp, vp, ql, kpl, vpl = inputs()
            snap = as_heads(kernels.paged_decode_attention_gather(
                ql, kpl, vpl, bt_d, ctx_d, exh, workspace=ws)).clone()
            check(f"host-epoch step {step}", snap, q, kp, vp)

        # 3) CUDA graph of two launches (one per slot) plus the copies that read them,
        #    replayed twice with new inputs written in place
        exg = PeerExchange(B, shard.n_q, D, torch.bfloat16)
        q, kp, vp, ql, kpl, vpl = inputs()
        ql2 = ql.clone()
        snaps = [torch.empty((B, Hq, D), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        for s_, qq in zip(snaps, (ql, ql2)):  # eager warm-up (workspace, slots 0 and 1)
            s_.copy_(as_heads(kernels.paged_decode_attention_gather(
                qq, kpl, vpl, bt_d, ctx_d, exg, workspace=ws)))
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for s_, qq in zip(snaps, (ql, ql2)):
                s_.copy_(as_heads(kernels.paged_decode_attention_gather(
                    qq, kpl, vpl, bt_d, ctx_d, exg, workspace=ws)))
        for rep in range(2):
            qa, kpa, vpa, qla, kpla, vpla = inputs()
            qb = torch.randn((B, Hq, D), generator=g).to(torch.bfloat16).to(dev)
            ql.copy_(qla)
            ql2.copy_(qb[:, shard.q_lo:shard.q_hi])
            kpl.copy_(kpla)
            vpl.copy_(vpla)
            graph.replay()
            check(f"graph replay {rep} slot 0", snaps[0].clone(), qa, kpa, vpa)
            check(f"graph replay {rep} slot 1", snaps[1].clone(), qb, kpa, vpa)
        torch.cuda.synchronize()
        del graph

        # 4) fewer KV heads than ranks: the KV head is replicated and its replicas split
        #    its query heads (C4 on 8 GPUs)
        hq2, hkv2 = 8, 1
        sh2 = head_shard(hq2, hkv2, world, rank)
        exr = PeerExchange(B, sh2.n_q, D, torch.bfloat16)
        for step in range(2):
            q, kp, vp, ql, kpl, vpl = inputs(hq2, hkv2)
            snap = as_heads(kernels.paged_decode_attention_gather(
                ql, kpl, vpl, bt_d, ctx_d, exr, workspace=ws), hq2).clone()
            check(f"replicated KV head step {step}", snap, q, kp, vp)
        with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
            f.write("ok" if ok else msg)
        dist.barrier()
        # 5) programmatic launch on: back-to-back gather launches may start while the
        #    previous one runs; each reads its epoch only after the programmatic wait
        kernels.set_programmatic_launch(True)
        try:
            for step in range(3):
                q, kp, vp, ql, kpl, vpl = inputs()
                snap = as_heads(kernels.paged_decode_attention_gather(
                    ql, kpl, vpl, bt_d, ctx_d, ex, workspace=ws)).clone()
                check(f"programmatic launch step {step}", snap, q, kp, vp)
        finally:
            kernels.set_programmatic_launch(False)
        for e in (ex, exh, exg, exr):
            e.close()
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
            f.write(traceback.format_exc())
        os._exit(3)


@pytest.mark.skipif(NGPU < 2, reason="needs at least two GPUs")
def test_peer_gather_equals_unsharded_and_nccl(tmp_path) -> None:
    import torch.multiprocessing as mp

    world = 2 if NGPU < 4 else (4 if NGPU < 8 else 8)
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
            p.join()
    msgs = [(tmp_path / f"rank{r}.txt").read_text() if (tmp_path / f"rank{r}.txt").exists()
            else "no result" for r in range(world)]
    assert all(m == "ok" for m in msgs), msgs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
