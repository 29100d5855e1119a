"""CPU check of the tcgen05 prefill kernel's addressing (csrc/paged_prefill_tc.cu).

The kernel has not run on a GPU yet. This restates its layout constants and index
arithmetic and checks, for every instantiated shape (head_dim 64/128, pages of 16/32)
and a sweep of launch shapes, that:
- every shared-memory offset it forms (Q, the K/V stages, TMA box destinations, P, the
  V zeroing of the last tile, the MMA descriptor start addresses) stays inside its region,
  and the regions fit the dynamic allocation it requests;
- each tile's expect-tx byte count equals the bytes its TMA boxes deliver;
- every page id it reads lies inside block_table[0, ceil(kv_len / S));
- the TMEM columns it uses fit the 256 it allocates.
The constants are restated here on purpose: a change on one side fails the check.
"""

from __future__ import annotations

import itertools
import pathlib
import re

import pytest

SRC = pathlib.Path(__file__).resolve().parent.parent / "plastic_infer_b200" / "csrc" / "paged_prefill_tc.cu"

KM = KN = 128
STAGES = 2
TMEM_COLS = 256
O_COL = 128


def cfg(D: int, S: int) -> dict:
    boxes = D // 64
    box_bytes = 128 * 128
    q_bytes = boxes * box_bytes
    kv_bytes = boxes * box_bytes
    stage = 2 * kv_bytes
    p_bytes = 2 * box_bytes
    smem = 1024 + q_bytes + STAGES * stage + p_bytes + (STAGES + 1) * 8 + 16
    return dict(boxes=boxes, box=box_bytes, q=q_bytes, kv=kv_bytes, stage=stage, p=p_bytes,
                pages_per_tile=KN // S, smem=smem)


def sw128_off(r: int, ch: int) -> int:
    return (ch >> 3) * (128 * 128) + r * 128 + (((ch & 7) ^ (r & 7)) << 4)


def test_constants_match_the_kernel_source() -> None:
    src = SRC.read_text()
    for name, val in (("kM", KM), ("kN", KN), ("kStages", STAGES)):
        assert re.search(rf"constexpr int {name} = {val};", src), name
    assert re.search(rf"constexpr uint32_t kTmemCols = {TMEM_COLS};", src)
    assert re.search(rf"constexpr uint32_t kOCol = {O_COL};", src)


@pytest.mark.parametrize("D,S", list(itertools.product((64, 128), (16, 32))))
def test_shared_memory_and_tmem_bounds(D: int, S: int) -> None:
    c = cfg(D, S)
    assert c["smem"] <= 227 * 1024
    q0, kv0 = 0, c["q"]
    p0 = kv0 + STAGES * c["stage"]
    bars0 = p0 + c["p"]
    slot0 = bars0 + (STAGES + 1) * 8
    assert slot0 + 4 <= c["smem"] - 1024  # after the 1024-byte alignment slack
    assert kv0 % 1024 == 0 and p0 % 1024 == 0 and c["stage"] % 1024 == 0
    # Q writes: rows < 128, 16-byte chunks < D / 8
    assert max(sw128_off(r, ch) for r in range(KM) for ch in range(D // 8)) + 16 <= c["q"]
    # P writes: 128 keys = 16 chunks per row
    assert max(sw128_off(r, ch) for r in range(KM) for ch in range(KN // 8)) + 16 <= c["p"]
    # TMA box destinations of one tile (K and V alike): box b, page pp
    for pp in range(c["pages_per_tile"]):
        for b in range(c["boxes"]):
            off = b * c["box"] + pp * S * 128
            assert off % 1024 == 0 and off + S * 128 <= c["kv"]
    # S = Q K^T descriptors: k step kk at box kk // 4, +32 B inside the 128-byte row
    for kk in range(D // 16):
        off = (kk >> 2) * c["box"] + (kk & 3) * 32
        assert off + 32 <= c["q"] and (off >> 4) < (1 << 14)
    # O += P V: P (K-major) as above over 128 keys; V (MN-major) steps 16 keys = 2048 B,
    # its second 64-column block one box further (the leading byte offset)
    for kk in range(KN // 16):
        assert (kk >> 2) * c["box"] + (kk & 3) * 32 + 32 <= c["p"]
        v_off = kk * 16 * 128
        assert v_off + 16 * 128 <= c["box"]
        assert v_off + (c["boxes"] - 1) * c["box"] + 16 * 128 <= c["kv"]
    # descriptors hold addresses >> 4 in 14 bits: the whole allocation must stay below 256 KB
    assert c["smem"] < (1 << 18)
    # TMEM: S in [0, 128), O in [128, 128 + D)
    assert KN <= O_COL and O_COL + D <= TMEM_COLS


@pytest.mark.parametrize("D,S", list(itertools.product((64, 128), (16, 32))))
@pytest.mark.parametrize("G", [1, 2, 4, 8, 16])
def test_page_reads_tiles_and_expect_tx(D: int, S: int, G: int) -> None:
    c = cfg(D, S)
    T = KM // G
    for q_len, kv_len, q_start, causal in [
        (1, 1, 0, True), (37, 37, 0, True), (300, 700, 400, True), (129, 129, 0, True),
        (40, 77, 0, False), (5, 3, 0, False), (4096, 4096, 0, True), (1024, 4096, 3072, True),
        (7, 0, 0, True), (200, 5000, 4800, True),
    ]:
        table_len = -(-kv_len // S)
        for qb in range(-(-q_len // T)):
            t0 = qb * T
            t_end = min(q_len, t0 + T)
            kv_hi = min(kv_len, q_start + t_end) if causal else kv_len
            n_tiles = -(-kv_hi // KN) if kv_hi > 0 else 0
            n_pages = -(-kv_hi // S)
            assert n_pages <= table_len
            for j in range(n_tiles):
                pg0 = j * c["pages_per_tile"]
                np_ = min(c["pages_per_tile"], n_pages - pg0)
                assert np_ >= 1 and pg0 + np_ <= n_pages
                # expect-tx bytes == what the boxes deliver (K and V, every box, every page)
                assert np_ * 2 * c["boxes"] * S * 128 == sum(
                    S * 128 for _ in range(np_) for _ in range(c["boxes"]) for _ in range(2))
                # last tile: V rows past the context are zeroed inside the V tile
                valid = min(KN, kv_hi - j * KN)
                assert 1 <= valid <= KN
                per_box = (KN - valid) * 8
                for cc in range(c["boxes"] * per_box):
                    b, rem = divmod(cc, per_box)
                    off = b * c["box"] + (valid + rem // 8) * 128 + (rem & 7) * 16
                    assert off + 16 <= c["kv"]
            # a row's visible keys never exceed what the CTA loaded
            for r in range(KM):
                tok = t0 + r // G
                lim = min(kv_len, q_start + tok + 1) if causal else kv_len
                if tok < q_len:
                    assert lim <= kv_hi
