"""KV-head sharding across ranks (row e), on CPU `gloo` ranks with the oracle.

Each rank holds only its KV heads' pools, attends its query heads with the oracle
(standing in for the kernel, which needs a GPU), and the all-gather assembles the
full [B, Hq, D] output; it must equal the unsharded oracle. Covers the even split
(Qwen3-8B: 8 KV heads on 2/4/8 ranks), replication (Qwen3-30B-A3B: 4 KV heads on 8
ranks), and a rank that fails before the collective (the others must error out,
not hang).
"""

from __future__ import annotations

import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from plastic_infer_b200.dist import head_shard, local_kv_rows, sharded_decode_attention


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(Hq: int, Hkv: int, seed: int = 0):
    rng = np.random.default_rng(seed)
    B, D, S = 3, 32, 4
    ctx = [5, 12, 1]
    npg = [-(-c // S) for c in ctx]
    P = sum(npg) + 1
    perm = rng.permutation(P)
    tables, cur = [], 0
    for n in npg:
        tables.append([int(x) for x in perm[cur:cur + n]])
        cur += n
    q = rng.standard_normal((B, Hq, D), dtype=np.float32)
    k = rng.standard_normal((P, Hkv, D, S), dtype=np.float32)
    v = rng.standard_normal((P, Hkv, D, S), dtype=np.float32)
    return q, k, v, tables, ctx, S


def _rank_main(rank: int, world: int, port: int, Hq: int, Hkv: int, out_dir: str,
               fail_rank: int) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    from oracle import paged_kv_oracle as orc

    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=10))
        q, k, v, tables, ctx, S = _problem(Hq, Hkv)
        shard = head_shard(Hq, Hkv, world, rank)
        kl = k[:, shard.kv_lo:shard.kv_hi]
        vl = v[:, shard.kv_lo:shard.kv_hi]
        # the rank's index-copy input is its own KV heads of the new rows
        rows = torch.arange(Hkv * 2, dtype=torch.float32).view(1, Hkv, 2)
        assert torch.equal(local_kv_rows(rows, shard)[0, :, 0],
                           torch.arange(shard.kv_lo, shard.kv_hi, dtype=torch.float32) * 2)

        def attend(q_local: torch.Tensor) -> torch.Tensor:
            if rank == fail_rank:
                raise RuntimeError("injected rank failure before the all-gather")
            return torch.from_numpy(orc.paged_attention_decode(q_local.numpy(), kl, vl, tables, ctx, S))

        full = sharded_decode_attention(torch.from_numpy(q), shard, attend)
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), full.numpy())
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(out_dir, f"rank{rank}.err"), "w") as f:
            f.write(traceback.format_exc())
        os._exit(3)


def _launch(world: int, Hq: int, Hkv: int, tmp_path, fail_rank: int = -1) -> list[int]:
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, Hq, Hkv, str(tmp_path), fail_rank))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            p.join()
    return [p.exitcode for p in procs]


@pytest.mark.parametrize("world,Hq,Hkv", [(2, 32, 8), (4, 32, 8), (8, 32, 8), (8, 32, 4), (2, 4, 2)])
def test_sharded_attention_equals_unsharded(world, Hq, Hkv, tmp_path) -> None:
    from oracle import paged_kv_oracle as orc

    codes = _launch(world, Hq, Hkv, tmp_path)
    errs = [f.read_text() for f in tmp_path.glob("*.err")]
    assert codes == [0] * world, errs
    q, k, v, tables, ctx, S = _problem(Hq, Hkv)
    ref = orc.paged_attention_decode(q, k, v, tables, ctx, S)
    for r in range(world):
        got = np.load(tmp_path / f"rank{r}.npy")
        np.testing.assert_allclose(got, ref, atol=1e-6, rtol=1e-6)


def test_failed_rank_makes_peers_error_not_hang(tmp_path) -> None:
    codes = _launch(2, 32, 8, tmp_path, fail_rank=1)
    assert codes[1] == 3 and "injected rank failure" in (tmp_path / "rank1.err").read_text()
    # the surviving rank's collective must end with an error (peer gone / timeout)
    assert codes[0] == 3, "rank 0 finished a collective its peer never joined"


def test_head_shard_rules() -> None:
    s = head_shard(32, 8, 8, 3)
    assert (s.kv_lo, s.kv_hi, s.q_lo, s.q_hi, s.replicas) == (3, 4, 12, 16, 1)
    s = head_shard(32, 4, 8, 5)   # Qwen3-30B-A3B on 8 GPUs: KV head 2 on ranks 4 and 5
    assert (s.kv_lo, s.kv_hi, s.q_lo, s.q_hi, s.replicas) == (2, 3, 20, 24, 2)
    with pytest.raises(ValueError):
        head_shard(32, 8, 3, 0)
    with pytest.raises(ValueError):
        head_shard(12, 4, 8, 0)
