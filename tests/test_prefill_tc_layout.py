"""CPU check of the tcgen05 prefill kernel's addressing (csrc/paged_prefill_tc.cu).

This restates the kernel's layout constants and index arithmetic and checks, for every
instantiated shape (head_dim 64/128, pages of 16/32) and a sweep of launch shapes, that:
- every shared-memory offset it forms (Q, the K and V rings, TMA box
  destinations, P, the V zeroing of the last tile, the MMA descriptor start addresses)
  stays inside its region, the regions fit the dynamic allocation it requests, and two
  CTAs of head_dim 128 fit on one SM (228 KB of shared memory, 1 KB reserved per CTA)
  while their TMEM columns fit the SM's 512;
- each load's expect-tx byte count equals the bytes its TMA boxes deliver;
- every page id it reads lies inside block_table[0, ceil(kv_len / S));
- the TMEM columns it uses fit the ones it allocates.
The constants are restated here on purpose: a change on one side fails the check.
"""

from __future__ import annotations

import itertools
import pathlib
import re

import pytest

SRC = pathlib.Path(__file__).resolve().parent.parent / "plastic_infer_b200" / "csrc" / "paged_prefill_tc.cu"

KM = 128
KN = 64
K_SLOTS = 2
V_SLOTS = 2
SLACK = 896
O_COL = 64
SM_SMEM = 228 * 1024
TMEM_PER_SM = 512


def cfg(D: int, S: int) -> dict:
    boxes = D // 64
    q_box = KM * 128
    kv_box = KN * 128
    q_bytes = boxes * q_box
    kv_bytes = boxes * kv_box
    p_bytes = KM * 128
    tmem_cols = 128 if O_COL + D <= 128 else 256
    layout = q_bytes + (K_SLOTS + V_SLOTS) * kv_bytes + p_bytes + 64
    smem = SLACK + layout
    return dict(boxes=boxes, q_box=q_box, kv_box=kv_box, q=q_bytes, kv=kv_bytes, p=p_bytes,
                pages_per_tile=KN // S, smem=smem, layout=layout, tmem_cols=tmem_cols)


def sw128_off(r: int, ch: int) -> int:
    return (ch >> 3) * (128 * 128) + r * 128 + (((ch & 7) ^ (r & 7)) << 4)


def test_constants_match_the_kernel_source() -> None:
    src = SRC.read_text()
    for name, val in (("kM", KM), ("kN", KN), ("kKSlots", K_SLOTS), ("kVSlots", V_SLOTS)):
        assert re.search(rf"constexpr int {name} = {val};", src), name
    assert re.search(rf"constexpr uint32_t kOCol = {O_COL};", src)
    assert re.search(rf"static constexpr int kSlack = {SLACK};", src)
    assert "kOCol + D <= 128 ? 128 : 256" in src
    assert "(kKSlots + kVSlots) * kKVBytes + kPBytes + kBarBytes" in src


@pytest.mark.parametrize("D,S", list(itertools.product((64, 128), (16, 32))))
def test_shared_memory_and_tmem_bounds(D: int, S: int) -> None:
    c = cfg(D, S)
    assert c["smem"] <= 227 * 1024
    # CTAs per SM by shared memory, and their TMEM never exceeds the SM's 512 columns (so
    # tcgen05.alloc never has to wait for another CTA's columns)
    ctas = SM_SMEM // (c["smem"] + 1024)
    assert ctas >= 2
    assert ctas * c["tmem_cols"] <= TMEM_PER_SM
    q0 = 0
    k0 = q0 + c["q"]
    v0 = k0 + K_SLOTS * c["kv"]
    p0 = v0 + V_SLOTS * c["kv"]
    bars0 = p0 + c["p"]
    assert bars0 + (K_SLOTS + V_SLOTS + 1) * 8 + 4 <= c["layout"]
    for off in (k0, v0, p0, c["kv"]):
        assert off % 1024 == 0
    # the layout fits after aligning any 128-byte aligned base up to 1024 bytes
    assert all((-base) % 1024 + c["layout"] <= c["smem"] for base in range(0, 4096, 128))
    # Q writes: rows < 128, 16-byte chunks < D / 8
    assert max(sw128_off(r, ch) for r in range(KM) for ch in range(D // 8)) + 16 <= c["q"]
    # P writes: 64 keys = 8 chunks per row, one box
    assert max(sw128_off(r, ch) for r in range(KM) for ch in range(KN // 8)) + 16 <= c["p"]
    # TMA box destinations of one K or V tile: box b, page pp
    for pp in range(c["pages_per_tile"]):
        for b in range(c["boxes"]):
            off = b * c["kv_box"] + pp * S * 128
            assert off % 1024 == 0 and off + S * 128 <= c["kv"]
    # S = Q K^T descriptors: k step kk at box kk // 4 (Q boxes 16 KB, K boxes 8 KB), +32 B
    for kk in range(D // 16):
        q_off = (kk >> 2) * c["q_box"] + (kk & 3) * 32
        k_off = (kk >> 2) * c["kv_box"] + (kk & 3) * 32
        assert q_off + 32 <= c["q"] and k_off + 32 <= c["kv"]
    # O += P V: P (K-major) over 64 keys in one box; V (MN-major) steps 16 keys = 2048 B,
    # its second 64-column block one box further (the leading byte offset)
    for kk in range(KN // 16):
        assert kk * 32 + 32 <= 128
        v_off = kk * 16 * 128
        assert v_off + 16 * 128 <= c["kv_box"]
        assert v_off + (c["boxes"] - 1) * c["kv_box"] + 16 * 128 <= c["kv"]
    # descriptors hold addresses >> 4 in 14 bits: the whole allocation must stay below 256 KB
    assert c["smem"] < (1 << 18)
    # TMEM: S in [0, 64), O in [64, 64 + D)
    assert KN <= O_COL and O_COL + D <= c["tmem_cols"]


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
        n_qblocks = -(-q_len // T)
        for bx in range(n_qblocks):
            qb = n_qblocks - 1 - bx if causal else bx   # heaviest block first when causal
            assert 0 <= qb < n_qblocks
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
                # expect-tx bytes of one K (or V) load == what its boxes deliver
                assert np_ * c["boxes"] * S * 128 == sum(
                    S * 128 for _ in range(np_) for _ in range(c["boxes"]))
                # last tile: V rows past the context are zeroed inside V(j)'s slot
                valid = min(KN, kv_hi - j * KN)
                assert 1 <= valid <= KN
                per_box = (KN - valid) * 8
                for cc in range(c["boxes"] * per_box):
                    b, rem = divmod(cc, per_box)
                    off = b * c["kv_box"] + (valid + rem // 8) * 128 + (rem & 7) * 16
                    assert off + 16 <= c["kv"]
            # a row's visible keys never exceed what the CTA loaded
            for r in range(KM):
                tok = t0 + r // G
                lim = min(kv_len, q_start + tok + 1) if causal else kv_len
                if tok < q_len:
                    assert lim <= kv_hi


def test_load_slots_phases_and_page_ids() -> None:
    # K(t) in slot t % 2, V(t) in V slot t % 2 (phase (t // 2) & 1). Tiles 0 and 1 load in
    # the prologue; after S(j) completes (and with it P V(j - 1)), K(j + 2) takes K(j)'s slot
    # and V(j + 1) takes V(j - 1)'s. Thread 0's page ids: ids_k = tile j + 1, ids_n = tile
    # j + 2 at the top of iteration j.
    for n in range(0, 12):
        k_issued = v_issued = min(2, n)
        ids_k, ids_n = 1, 2
        for j in range(n):
            assert j < k_issued and j < v_issued  # tile j's K and V were issued before its waits
            if k_issued < n and k_issued == j + K_SLOTS:
                assert k_issued % K_SLOTS == j % K_SLOTS   # K(j) consumed by S(j): done
                assert ids_n == k_issued
                k_issued += 1
            if j >= 1 and v_issued < n and v_issued == j + 1:
                # V(j + 1)'s slot held V(j - 1), read by P V(j - 1): done before S(j)
                assert v_issued % V_SLOTS == (j - 1) % V_SLOTS
                assert ids_k == v_issued
                v_issued += 1
            ids_k, ids_n = ids_n, j + 3
        assert k_issued == n and v_issued == n
