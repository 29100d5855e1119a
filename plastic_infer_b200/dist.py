"""Multi-GPU paged decode by KV-head sharding (one process per GPU).

The reference is single-GPU (no torch.distributed anywhere). Here the KV path splits
across N ranks by KV head, the natural partition of GQA attention:

  * rank r owns KV heads [r*Hkv/N, (r+1)*Hkv/N) and their query heads; its page pools
    hold only those heads ([P, Hkv/N, page_size, head_dim]). Page ids, block tables,
    context lengths and slot mappings are the same on every rank, so the host
    allocator runs unchanged and each rank's index-copy writes its own heads.
  * When Hkv < N (e.g. 4 KV heads on 8 GPUs), each KV head is replicated on N/Hkv
    ranks and those ranks split its G query heads between them
    (the reference's div_even(..., allow_replicate) rule, src/plastic_infer/utils/__init__.py:18-24);
    each replica's index-copy writes its own copy of the head.
  * the only exchange is one all-gather per layer of the per-rank attention outputs
    [B, Hq/N, D] into [N, B, Hq/N, D] before o_proj. Because rank r's query heads are
    the r-th contiguous block, the gathered tensor is already [B, Hq, D] after one
    transpose (or none, if o_proj's input columns are permuted once at load time).

The compute function is passed in, so the same sharding logic runs on CPU `gloo`
ranks in tests (with the oracle) and on NCCL ranks with the kernels.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    kv_lo: int      # first KV head held by this rank
    kv_hi: int
    q_lo: int       # first query head computed by this rank
    q_hi: int
    replicas: int   # ranks holding each KV head (1 = no replication)

    @property
    def n_kv(self) -> int:
        return self.kv_hi - self.kv_lo

    @property
    def n_q(self) -> int:
        return self.q_hi - self.q_lo


def head_shard(n_q_heads: int, n_kv_heads: int, world: int, rank: int) -> HeadShard:
    """This rank's KV and query heads; raises if the heads do not divide evenly."""
    if n_q_heads % n_kv_heads:
        raise ValueError("n_q_heads must be a multiple of n_kv_heads")
    if n_q_heads % world:
        raise ValueError(f"{n_q_heads} query heads do not split over {world} ranks")
    group = n_q_heads // n_kv_heads
    nq = n_q_heads // world
    if n_kv_heads % world == 0:
        nkv = n_kv_heads // world
        return HeadShard(rank, world, rank * nkv, (rank + 1) * nkv, rank * nq, (rank + 1) * nq, 1)
    if world % n_kv_heads:
        raise ValueError(f"{n_kv_heads} KV heads neither split over nor replicate onto {world} ranks")
    rep = world // n_kv_heads
    if group % rep:
        raise ValueError("query heads of a KV head do not split over its replicas")
    kv = rank // rep
    return HeadShard(rank, world, kv, kv + 1, rank * nq, (rank + 1) * nq, rep)


def local_q(q: torch.Tensor, shard: HeadShard) -> torch.Tensor:
    """This rank's query heads of q [B, Hq, D]."""
    return q[:, shard.q_lo:shard.q_hi]


def local_kv_rows(kv_new: torch.Tensor, shard: HeadShard) -> torch.Tensor:
    """This rank's KV heads of new rows [B, Hkv, D] (for the index-copy)."""
    return kv_new[:, shard.kv_lo:shard.kv_hi]


def gather_heads(local_out: torch.Tensor, shard: HeadShard,
                 group: dist.ProcessGroup | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather per-rank outputs [B, Hq/N, D] into [B, Hq, D] (rank-major heads)."""
    B, nq, D = local_out.shape
    # rank-major [world * B, nq, D]: every backend splits the output along dim 0
    buf = torch.empty((shard.world * B, nq, D), dtype=local_out.dtype, device=local_out.device)
    dist.all_gather_into_tensor(buf, local_out.contiguous(), group=group)
    full = buf.view(shard.world, B, nq, D).permute(1, 0, 2, 3).reshape(B, shard.world * nq, D)
    if out is not None:
        out.copy_(full)
        return out
    return full


def sharded_decode_attention(q: torch.Tensor, shard: HeadShard,
                             attend: Callable[[torch.Tensor], torch.Tensor],
                             group: dist.ProcessGroup | None = None) -> torch.Tensor:
    """Attention of q [B, Hq, D] with this rank's shard, gathered to [B, Hq, D].

    `attend(q_local)` runs this rank's attention over its own pools (the
    paged_decode_attention kernel on GPU) and returns [B, Hq/N, D].
    """
    return gather_heads(attend(local_q(q, shard).contiguous()), shard, group)
