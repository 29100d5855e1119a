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


# ---------------------------------------------------------------------------------
# Peer exchange: the all-gather fused into the attention kernel (NVLink peer stores)
# ---------------------------------------------------------------------------------

import ctypes  # noqa: E402

_IPC_HANDLE_BYTES = 64
_cudaIpcMemLazyEnablePeerAccess = 1


class _IpcHandle(ctypes.Structure):
    # c_ubyte, not c_char: a c_char array reads back as a C string cut at the first NUL
    _fields_ = [("reserved", ctypes.c_ubyte * _IPC_HANDLE_BYTES)]


def _cudart() -> ctypes.CDLL:
    """The CUDA runtime already loaded by torch (same SONAME), via ctypes."""
    import torch  # noqa: F401  (makes sure torch's libcudart is loaded first)

    lib = ctypes.CDLL("libcudart.so.12")
    lib.cudaMalloc.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t]
    lib.cudaFree.argtypes = [ctypes.c_void_p]
    lib.cudaMemset.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t]
    lib.cudaIpcGetMemHandle.argtypes = [ctypes.POINTER(_IpcHandle), ctypes.c_void_p]
    lib.cudaIpcOpenMemHandle.argtypes = [ctypes.POINTER(ctypes.c_void_p), _IpcHandle, ctypes.c_uint]
    lib.cudaIpcCloseMemHandle.argtypes = [ctypes.c_void_p]
    return lib


def _ck(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed with cudaError {rc}")


class _DevArray:
    """__cuda_array_interface__ view of raw device memory (for torch.as_tensor)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str) -> None:
        self.__cuda_array_interface__ = dict(shape=shape, typestr=typestr, data=(ptr, False),
                                             version=3, strides=None)


class PeerExchange:
    """Gathered-output buffers that every rank maps, for pi_paged_decode_attn_gather.

    Each rank cudaMallocs `slots` gathered-output buffers of [world, B, Hq/N, D] plus a
    flag array, shares them with CUDA IPC, and opens every peer's (NVLink peer access).
    A launch completes only once every rank's slice of it has landed here, so the
    gathered buffer can be read by whatever follows on the stream. Slots alternate per
    launch so that a rank one launch ahead never overwrites an output a slower peer is
    still reading (two slots suffice).

    With `device_epochs` (the default) the epochs live in a launch counter in this
    rank's buffer and the kernel advances it itself, so the arguments of the i-th
    launch of a step are the same every step: a step of a multiple of `slots`
    launches can be captured in a CUDA graph. Otherwise the host passes the epochs.
    The per-slot argument blocks and output views are built once here, keeping the
    per-launch host work to the kernel call.
    """

    def __init__(self, batch: int, q_heads_local: int, head_dim: int, dtype, group=None,
                 slots: int = 2, device_epochs: bool = True) -> None:
        import torch

        from . import _capi

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("at most 8 ranks (one NVSwitch domain)")
        self.dtype = dtype
        self.shape = (self.world * batch, q_heads_local, head_dim)
        self.elem = torch.tensor([], dtype=dtype).element_size()
        self.slot_elems = self.world * batch * q_heads_local * head_dim
        self.rank_stride = batch * q_heads_local * head_dim
        self.slots = slots
        slot_bytes = (self.slot_elems * self.elem + 255) // 256 * 256
        self.flag_off = slot_bytes * slots
        self.nbytes = self.flag_off + 256
        cu = _cudart()
        self._cu = cu
        base = ctypes.c_void_p()
        _ck(cu.cudaMalloc(ctypes.byref(base), self.nbytes), "cudaMalloc")
        _ck(cu.cudaMemset(base, 0, self.nbytes), "cudaMemset")
        self.base = base.value
        h = _IpcHandle()
        _ck(cu.cudaIpcGetMemHandle(ctypes.byref(h), base), "cudaIpcGetMemHandle")
        handles: list = [None] * self.world
        dist.all_gather_object(handles, ctypes.string_at(ctypes.addressof(h), _IPC_HANDLE_BYTES),
                               group=group)
        self.ptrs: list[int] = []
        for r, hb in enumerate(handles):
            if r == self.rank:
                self.ptrs.append(self.base)
                continue
            peer = ctypes.c_void_p()
            hr = _IpcHandle()
            ctypes.memmove(ctypes.byref(hr), hb, _IPC_HANDLE_BYTES)
            _ck(cu.cudaIpcOpenMemHandle(ctypes.byref(peer), hr, _cudaIpcMemLazyEnablePeerAccess),
                "cudaIpcOpenMemHandle")
            self.ptrs.append(peer.value)
        self.slot_bytes = slot_bytes
        # flags: one word per rank at flag_off; this rank's launch counter after them
        self.counter_off = self.flag_off + 4 * _capi.MAX_PEERS
        self.device_epochs = device_epochs
        self.epoch = 0      # host epochs (device_epochs=False)
        self.calls = 0      # launches issued from the host (slot rotation)
        self.args = []
        for slot in range(slots):
            g = _capi.PeerGather()
            for r in range(self.world):
                g.peer_out[r] = self.ptrs[r] + slot * slot_bytes
                g.peer_flags[r] = self.ptrs[r] + self.flag_off
            g.rank, g.world, g.rank_stride = self.rank, self.world, self.rank_stride
            g.launch_counter = self.base + self.counter_off if device_epochs else None
            self.args.append(g)
        self.views = [self._slot_view(s) for s in range(slots)]
        dist.barrier(group=group)

    def _slot_view(self, slot: int):
        import torch

        typestr = {2: "<f2", 4: "<f4"}[self.elem]
        t = torch.as_tensor(_DevArray(self.base + slot * self.slot_bytes,
                                      (self.slot_elems,), typestr), device="cuda")
        return t.view(self.dtype).view(self.shape) if self.dtype != t.dtype else t.view(self.shape)

    def slot_tensor(self, slot: int):
        """This rank's local gathered buffer of `slot` as [world * B, Hq/N, D]."""
        return self.views[slot]

    def next_launch(self):
        """(slot, argument block) of the next gather launch; advances the rotation."""
        slot = self.calls % self.slots
        self.calls += 1
        g = self.args[slot]
        if not self.device_epochs:
            self.epoch += 1
            g.epoch = self.epoch
        return slot, g

    def close(self) -> None:
        if self.base is None:
            return
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                self._cu.cudaIpcCloseMemHandle(ctypes.c_void_p(p))
        self._cu.cudaFree(ctypes.c_void_p(self.base))
        self.base = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass
