"""GPU parity of the fused decode prologue (pi_decode_prologue).

One launch applies QK-norm (optional) and RoPE to the step's q and k rows and writes the
new K/V rows at their slots. Checked against:
- the reference's own qk_norm + rope_positions outputs (golden prologue.npz, fp32 table)
  in fp32, within 2e-5;
- the oracle on bf16 / f16 inputs and pools, within one rounding to the pool dtype
  (|err| <= 1e-2 + 8e-3 |ref|);
- V rows copied bit for bit, nothing else in the pools touched.
Also: strided slices of one fused QKV output, padding and out-of-range slots, and the
prologue followed by decode attention against the oracle.
"""

from __future__ import annotations

import pathlib

import numpy as np
import pytest
import torch

from oracle import paged_kv_oracle as orc
from plastic_infer_b200 import _capi, kernels
from tests.golden.inputs import PROLOGUE_CASES, prologue_inputs

pytestmark = pytest.mark.gpu
GOLD = pathlib.Path(__file__).resolve().parent / "golden"
DEV = torch.device("cuda", 0)
_T = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _pools(Hkv: int, D: int, dtype: torch.dtype, P: int = 40, S: int = 16):
    kp = torch.zeros((P, Hkv, S, D), dtype=dtype, device=DEV)
    return kp, torch.zeros_like(kp)


def _slots(B: int, P: int = 40, S: int = 16, seed: int = 0) -> np.ndarray:
    return np.random.default_rng(seed).permutation(P * S)[:B].astype(np.int64)


def _rows_at(pool: torch.Tensor, slots: np.ndarray) -> np.ndarray:
    S = pool.shape[2]
    s = torch.from_numpy(slots).to(DEV)
    return pool[s // S, :, s % S, :].float().cpu().numpy()  # [B, Hkv, D]


def _run(x: dict, case: dict, in_dt: str, pool_dt: str, slots: np.ndarray):
    D, Hkv = case["D"], case["Hkv"]
    kp, vp = _pools(Hkv, D, _T[pool_dt])
    q = torch.from_numpy(x["q"]).to(_T[in_dt]).to(DEV)
    k = torch.from_numpy(x["k"]).to(_T[in_dt]).to(DEV)
    v = torch.from_numpy(x["v"]).to(_T[in_dt]).to(DEV)
    qw = kw = None
    if case["qk_norm"]:
        qw = torch.from_numpy(x["q_norm_w"]).to(DEV)
        kw = torch.from_numpy(x["k_norm_w"]).to(DEV)
    out = kernels.decode_prologue(q, k, v, torch.from_numpy(x["positions"]).to(DEV),
                                  kernels.rope_inv_freq(D, case["base"], DEV),
                                  torch.from_numpy(slots).to(DEV), kp, vp, qw, kw)
    torch.cuda.synchronize()
    return out, kp, vp, (q, k, v, qw, kw)


@pytest.mark.parametrize("case", PROLOGUE_CASES, ids=[c["name"] for c in PROLOGUE_CASES])
def test_prologue_matches_reference_golden_fp32(case: dict) -> None:
    g = np.load(GOLD / "prologue.npz")
    n = case["name"]
    x = prologue_inputs(case)
    slots = _slots(case["B"])
    out, kp, vp, _ = _run(x, case, "f32", "f32", slots)
    np.testing.assert_allclose(out.cpu().numpy(), g[n + "__q"], rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(_rows_at(kp, slots), g[n + "__k"], rtol=2e-5, atol=2e-5)
    assert np.array_equal(_rows_at(vp, slots), x["v"])
    # nothing else written
    S = kp.shape[2]
    mask = torch.ones(kp.shape[0] * S, dtype=torch.bool)
    mask[torch.from_numpy(slots)] = False
    rest = kp.permute(0, 2, 1, 3).reshape(-1, kp.shape[1], kp.shape[3])[mask.to(DEV)]
    assert int(torch.count_nonzero(rest)) == 0


@pytest.mark.parametrize("in_dt,pool_dt", [("bf16", "bf16"), ("f16", "f16"), ("f32", "bf16")])
@pytest.mark.parametrize("case", PROLOGUE_CASES, ids=[c["name"] for c in PROLOGUE_CASES])
def test_prologue_half_precision_vs_oracle(case: dict, in_dt: str, pool_dt: str) -> None:
    x = prologue_inputs(case)
    slots = _slots(case["B"], seed=1)
    out, kp, vp, (q, k, v, qw, kw) = _run(x, case, in_dt, pool_dt, slots)
    # the oracle sees exactly the values the kernel read
    inv = kernels.rope_inv_freq(case["D"], case["base"]).numpy()
    rq, rk, _ = orc.decode_prologue(q.float().cpu().numpy(), k.float().cpu().numpy(), None,
                                    x["positions"], inv,
                                    None if qw is None else qw.to(q.dtype).float().cpu().numpy(),
                                    None if kw is None else kw.to(q.dtype).float().cpu().numpy())
    for got, ref in ((out.float().cpu().numpy(), rq), (_rows_at(kp, slots), rk)):
        err = np.abs(got - ref)
        assert (err <= 1e-2 + 8e-3 * np.abs(ref)).all(), f"max err {err.max():.3e}"
    # V: the same bits (a conversion only when the input dtype differs from the pool's)
    assert torch.equal(torch.from_numpy(_rows_at(vp, slots)), v.to(_T[pool_dt]).float().cpu())


def test_prologue_fused_qkv_slices_padding_and_bad_slots() -> None:
    B, Hq, Hkv, D, S, P = 5, 8, 2, 128, 16, 20
    g = torch.Generator(device=DEV).manual_seed(3)
    qkv = torch.randn((B, (Hq + 2 * Hkv) * D), dtype=torch.bfloat16, device=DEV, generator=g)
    q = qkv[:, :Hq * D].view(B, Hq, D)
    k = qkv[:, Hq * D:(Hq + Hkv) * D].view(B, Hkv, D)
    v = qkv[:, (Hq + Hkv) * D:].view(B, Hkv, D)
    pos = torch.tensor([5, 0, 300, 17, 1000], dtype=torch.int64, device=DEV)
    slots = torch.tensor([3, -1, 77, P * S + 4, 150], dtype=torch.int64, device=DEV)
    kp = torch.zeros((P, Hkv, S, D), dtype=torch.bfloat16, device=DEV)
    vp = torch.zeros_like(kp)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    inv = kernels.rope_inv_freq(D, 1e6, DEV)
    out = kernels.decode_prologue(q, k, v, pos, inv, slots, kp, vp, err=err)
    # reference: the same inputs made contiguous
    kp2, vp2 = torch.zeros_like(kp), torch.zeros_like(kp)
    ok_slots = torch.tensor([3, -1, 77, -1, 150], dtype=torch.int64, device=DEV)
    out2 = kernels.decode_prologue(q.contiguous(), k.contiguous(), v.contiguous(), pos, inv,
                                   ok_slots, kp2, vp2)
    torch.cuda.synchronize()
    assert int(err.item()) == _capi.PI_ERR_SLOT_RANGE
    assert torch.equal(out, out2)
    assert torch.equal(kp, kp2) and torch.equal(vp, vp2)
    assert int(torch.count_nonzero(kp)) == 3 * Hkv * D  # slots 3, 77, 150 only


def test_prologue_then_attention_vs_oracle() -> None:
    # one decode step of the 8B head shape: prologue writes the new rows, attention reads
    # them at position ctx - 1
    B, Hq, Hkv, D, S = 6, 32, 8, 128, 16
    rng = np.random.default_rng(9)
    ctx = np.array([1, 16, 17, 200, 513, 64])
    npg = -(-ctx // S)
    P = int(npg.sum()) + 3
    perm = rng.permutation(P)
    tables, cur = [], 0
    for n in npg:
        tables.append([int(t) for t in perm[cur:cur + n]])
        cur += n
    lk = orc.f32_to_bf16_bits(rng.standard_normal((P, Hkv, D, S), dtype=np.float32))
    lv = orc.f32_to_bf16_bits(rng.standard_normal((P, Hkv, D, S), dtype=np.float32))
    kp = torch.from_numpy(lk.view(np.int16)).view(torch.bfloat16).permute(0, 1, 3, 2).contiguous().to(DEV)
    vp = torch.from_numpy(lv.view(np.int16)).view(torch.bfloat16).permute(0, 1, 3, 2).contiguous().to(DEV)
    q = torch.randn((B, Hq, D), dtype=torch.bfloat16, device=DEV)
    k = torch.randn((B, Hkv, D), dtype=torch.bfloat16, device=DEV)
    v = torch.randn((B, Hkv, D), dtype=torch.bfloat16, device=DEV)
    pos = ctx - 1
    slots = np.array([orc.slot_of(t, int(c) - 1, S) for t, c in zip(tables, ctx)], dtype=np.int64)
    inv = kernels.rope_inv_freq(D, 1e6, DEV)
    qr = kernels.decode_prologue(q, k, v, torch.from_numpy(pos).to(DEV), inv,
                                 torch.from_numpy(slots).to(DEV), kp, vp)
    bt = torch.zeros((B, int(npg.max())), dtype=torch.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
    out = kernels.paged_decode_attention(qr, kp, vp, bt.to(DEV),
                                         torch.from_numpy(ctx.astype(np.int32)).to(DEV))
    torch.cuda.synchronize()
    # oracle: rope in fp32, one bf16 rounding of q and k as the kernel stores them
    oq, ok, _ = orc.decode_prologue(q.float().cpu().numpy(), k.float().cpu().numpy(), None, pos,
                                    inv.cpu().numpy())
    oq_b = orc.f32_to_bf16_bits(oq)
    ok_b = orc.f32_to_bf16_bits(ok)
    orc.write_kv_slots(lk, lv, ok_b, orc.f32_to_bf16_bits(v.float().cpu().numpy()), slots, S)
    # the pool K rows the kernel wrote equal the oracle's rounding (one rounding each side;
    # allow one bf16 ulp where fp32 rounding of cos/sin lands on the other side)
    got_k = kp.permute(0, 1, 3, 2).contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    diff = np.abs(orc.bf16_bits_to_f32(got_k) - orc.bf16_bits_to_f32(lk))
    assert (diff <= 8e-3 * np.abs(orc.bf16_bits_to_f32(lk)) + 1e-6).all()
    ref = orc.paged_attention_decode(orc.bf16_bits_to_f32(oq_b), orc.bf16_bits_to_f32(got_k),
                                     orc.bf16_bits_to_f32(lv), tables, list(ctx), S)
    o = out.float().cpu().numpy()
    err = np.abs(o - ref)
    assert (err <= 2e-2 + 1e-2 * np.abs(ref)).all(), f"max err {err.max():.3e}"
    # and q went through the same rounding
    assert np.abs(qr.float().cpu().numpy() - orc.bf16_bits_to_f32(oq_b)).max() <= 8e-3 * 4
