"""Programmatic dependent launch (pi_set_programmatic_launch) keeps every result.

With the switch on, each index-copy and attention kernel lets the next kernel on the
stream launch early. The attention computes its work split and fetches its first page
ids while the previous kernel finishes, and it waits for that kernel before it touches
q, the pools or its outputs. A decode-step sequence (index-copy of the new rows, then
attention over pages that include those rows, layer after layer) must give the same
bits with the switch on as with it off. This holds run eagerly and captured in a CUDA
graph. So must back-to-back attention launches that share one workspace, whose
counters the previous launch resets at its very end.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from plastic_infer_b200 import kernels

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _step_inputs(L: int = 6, B: int = 24, Hq: int = 32, Hkv: int = 8, D: int = 128, S: int = 16):
    rng = np.random.default_rng(11)
    ctx = rng.integers(1, 1500, size=B)
    ctx[3] = 0  # an empty request
    npg = (ctx + S - 1) // S
    per_layer = int(npg.sum())
    P = per_layer * L + 8
    perm = rng.permutation(P).astype(np.int32)
    bt = np.zeros((L, B, max(1, int(npg.max()))), np.int32)
    cur = 0
    for l in range(L):
        for b in range(B):
            bt[l, b, :npg[b]] = perm[cur:cur + npg[b]]
            cur += npg[b]
    # the step's new row of request b sits at its last context position
    last = np.maximum(ctx - 1, 0)
    slots = bt[np.arange(L)[:, None], np.arange(B)[None, :], last[None, :] // S] * S + last % S
    slots[:, 3] = -1  # the empty request appends nothing
    g = torch.Generator(device=DEV).manual_seed(5)
    return dict(
        kp=torch.randn((P, Hkv, S, D), dtype=torch.bfloat16, device=DEV, generator=g),
        vp=torch.randn((P, Hkv, S, D), dtype=torch.bfloat16, device=DEV, generator=g),
        q=torch.randn((L, B, Hq, D), dtype=torch.bfloat16, device=DEV, generator=g),
        kn=torch.randn((L, B, Hkv, D), dtype=torch.bfloat16, device=DEV, generator=g),
        vn=torch.randn((L, B, Hkv, D), dtype=torch.bfloat16, device=DEV, generator=g),
        bt=torch.from_numpy(bt).to(DEV),
        slots=torch.from_numpy(slots.astype(np.int64)).to(DEV),
        ctx=torch.from_numpy(ctx.astype(np.int32)).to(DEV),
    )


def _run_step(x: dict, out: torch.Tensor, ws: kernels.Workspace) -> None:
    for l in range(x["q"].shape[0]):
        kernels.kv_index_copy(x["kp"], x["vp"], x["kn"][l], x["vn"][l], x["slots"][l])
        kernels.paged_decode_attention(x["q"][l], x["kp"], x["vp"], x["bt"][l], x["ctx"],
                                       out=out[l], workspace=ws)


def _reference() -> tuple[torch.Tensor, dict]:
    kernels.set_programmatic_launch(False)
    x = _step_inputs()
    out = torch.empty_like(x["q"])
    _run_step(x, out, kernels.Workspace(DEV))
    torch.cuda.synchronize()
    return out, x


def test_decode_step_bit_identical_with_programmatic_launch() -> None:
    ref, xr = _reference()
    try:
        kernels.set_programmatic_launch(True)
        # eager
        x = _step_inputs()
        out = torch.empty_like(x["q"])
        ws = kernels.Workspace(DEV)
        _run_step(x, out, ws)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        assert torch.equal(x["kp"], xr["kp"]) and torch.equal(x["vp"], xr["vp"])
        # CUDA graph of the whole step, replayed on fresh pools
        x = _step_inputs()
        out = torch.empty_like(x["q"])
        kp0, vp0 = x["kp"].clone(), x["vp"].clone()
        _run_step(x, out, ws)  # first launches encode the TMA descriptors
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            _run_step(x, out, ws)
        for _ in range(2):
            x["kp"].copy_(kp0)
            x["vp"].copy_(vp0)
            out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, ref)
        del graph
    finally:
        kernels.set_programmatic_launch(False)


def test_back_to_back_attention_with_programmatic_launch() -> None:
    x = _step_inputs(L=8)
    ws = kernels.Workspace(DEV)
    outs = {}
    for on in (False, True):
        kernels.set_programmatic_launch(on)
        try:
            out = torch.empty_like(x["q"])
            for _ in range(3):
                for l in range(x["q"].shape[0]):
                    kernels.paged_decode_attention(x["q"][l], x["kp"], x["vp"], x["bt"][l],
                                                   x["ctx"], out=out[l], workspace=ws)
            torch.cuda.synchronize()
            outs[on] = out
        finally:
            kernels.set_programmatic_launch(False)
    assert torch.equal(outs[True], outs[False])
