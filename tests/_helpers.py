"""Conversions shared by the GPU parity tests (numpy oracle <-> torch device tensors)."""

from __future__ import annotations

import numpy as np
import torch

from oracle.paged_kv_oracle import bf16_bits_to_f32

_TORCH = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def torch_dtype(name: str) -> torch.dtype:
    return _TORCH[name]


def from_bits(bits: np.ndarray) -> torch.Tensor:
    """uint16 bf16 bit patterns -> torch.bfloat16 (CPU), bit-exact."""
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def to_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def host_tensor(values: np.ndarray, dtype: str, bits: np.ndarray | None = None) -> torch.Tensor:
    if dtype == "bf16":
        return from_bits(bits if bits is not None else _round_bits(values))
    return torch.from_numpy(np.ascontiguousarray(values)).to(_TORCH[dtype])


def _round_bits(values: np.ndarray) -> np.ndarray:
    from oracle.paged_kv_oracle import f32_to_bf16_bits

    return f32_to_bf16_bits(values)


def physical_from_logical(logical: torch.Tensor) -> torch.Tensor:
    """[P, H, D, S] -> contiguous [P, H, S, D]."""
    return logical.permute(0, 1, 3, 2).contiguous()


def logical_np(phys: torch.Tensor) -> np.ndarray:
    """Physical device pool -> logical [P, H, D, S] numpy (bits for bf16, values otherwise)."""
    lg = phys.detach().permute(0, 1, 3, 2).contiguous().cpu()
    if lg.dtype == torch.bfloat16:
        return lg.view(torch.int16).numpy().view(np.uint16)
    return lg.numpy()


def logical_f32(phys: torch.Tensor) -> np.ndarray:
    """Physical device pool -> logical [P, H, D, S] float32 numpy values."""
    return phys.detach().permute(0, 1, 3, 2).float().contiguous().cpu().numpy()


def allclose_report(out: np.ndarray, ref: np.ndarray, atol: float, rtol: float) -> str:
    err = np.abs(out - ref)
    bad = err > atol + rtol * np.abs(ref)
    return (f"max abs err {err.max():.3e}, violations {int(bad.sum())} / {bad.size}, "
            f"max |ref| {np.abs(ref).max():.3f}")


def assert_close(out: np.ndarray, ref: np.ndarray, atol: float, rtol: float) -> None:
    out = np.asarray(out, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    assert np.isfinite(out).all(), "non-finite output"
    ok = np.abs(out - ref) <= atol + rtol * np.abs(ref)
    assert ok.all(), allclose_report(out, ref, atol, rtol)


__all__ = ["assert_close", "bf16_bits_to_f32", "from_bits", "host_tensor", "logical_f32",
           "oracle_decode_by_request",
           "logical_np", "physical_from_logical", "to_bits", "torch_dtype"]


def oracle_decode_by_request(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                             tables: list[list[int]], ctx: list[int], page_size: int,
                             requests: list[int] | None = None) -> np.ndarray:
    """Oracle decode attention, one request at a time, reading only that request's pages.

    Physical device pools [P, H, S, D] of any size (a full 8B-shape layer is ~0.6 GB per
    pool): each request's pages are gathered on the device and widened to fp32 on the
    host, so host memory stays at one request's context. Returns [len(requests), Hq, D].
    """
    from oracle import paged_kv_oracle as orc

    reqs = list(range(len(ctx))) if requests is None else list(requests)
    qf = q.float().cpu().numpy()
    out = np.zeros((len(reqs), q.shape[1], q.shape[2]), dtype=np.float32)
    for i, b in enumerate(reqs):
        n = int(ctx[b])
        if n <= 0:
            continue
        npg = -(-n // page_size)
        ids = torch.tensor(tables[b][:npg], dtype=torch.int64, device=k_pool.device)
        kb = logical_f32(k_pool.index_select(0, ids))
        vb = logical_f32(v_pool.index_select(0, ids))
        out[i] = orc.paged_attention_decode(qf[b:b + 1], kb, vb, [list(range(npg))], [n],
                                            page_size)[0]
    return out
