"""CPU check of the tcgen05 prefill kernel's addressing (csrc/paged_prefill_tc.cu).

This restates the kernel's layout constants and index arithmetic and checks, for every
instantiated shape (head_dim 64/128, pages of 16/32) and a sweep of launch shapes, that:
- every shared-memory offset it forms (Q, the K and V rings, TMA box destinations, the V
  zeroing of the last tile, the MMA descriptor start addresses, the output staging)
  stays inside its region, the regions fit the dynamic allocation it requests, and two
  CTAs of head_dim 128 fit on one SM (228 KB of shared memory, 1 KB reserved per CTA)
  while their TMEM columns fit the SM's 512;
- each load's expect-tx byte count equals the bytes its TMA boxes deliver;
- every page id it reads lies inside block_table[0, ceil(kv_len / S));
- the TMEM columns it uses fit the ones it allocates, P(t) lies inside S(t)'s buffer, and
  the P V MMA's A-operand columns stay inside P;
- the warp-specialized protocol (load warp, MMA thread, 4 softmax warps over mbarriers)
  cannot deadlock and never reuses a buffer early, under random completion orders.
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
SLACK = 768
O_COL = 128
TMEM_COLS = 256
BAR_BYTES = 144
SM_SMEM = 228 * 1024
TMEM_PER_SM = 512


def cfg(D: int, S: int) -> dict:
    boxes = D // 64
    q_box = KM * 128
    kv_box = KN * 128
    q_bytes = boxes * q_box
    kv_bytes = boxes * kv_box
    layout = q_bytes + (K_SLOTS + V_SLOTS) * kv_bytes + BAR_BYTES
    smem = SLACK + layout
    launch = max(smem, 80 * 1024)
    return dict(boxes=boxes, q_box=q_box, kv_box=kv_box, q=q_bytes, kv=kv_bytes,
                pages_per_tile=KN // S, smem=smem, launch=launch, layout=layout)


def sw128_off(r: int, ch: int) -> int:
    return (ch >> 3) * (128 * 128) + r * 128 + (((ch & 7) ^ (r & 7)) << 4)


def test_constants_match_the_kernel_source() -> None:
    src = SRC.read_text()
    for name, val in (("kM", KM), ("kN", KN), ("kKSlots", K_SLOTS), ("kVSlots", V_SLOTS)):
        assert re.search(rf"constexpr int {name} = {val};", src), name
    assert re.search(rf"constexpr uint32_t kOCol = {O_COL};", src)
    assert re.search(rf"constexpr uint32_t kTmemCols = {TMEM_COLS};", src)
    assert re.search(rf"static constexpr int kSlack = {SLACK};", src)
    assert re.search(rf"static constexpr int kBarBytes = {BAR_BYTES};", src)
    assert "kSmem > 80 * 1024 ? kSmem : 80 * 1024" in src
    assert "(kKSlots + kVSlots) * kKVBytes + kBarBytes" in src
    # P V reads P from TMEM: tile t's P over the first 32 columns of S(t)'s buffer, K step kk
    # at 8 columns (16 bf16/f16 values) per MMA
    assert "umma_f16_ts(tmem + kOCol, tmem + static_cast<uint32_t>(kN * (u % 2) + 8 * kk)" in src
    assert "tmem_st32(t_row + static_cast<uint32_t>(kN * sb), pf);" in src
    # P ready is two barriers by tile parity (the simulation below needs them)
    assert "mbar_arrive(bar(kPFull + sb));" in src
    assert "mbar_wait_bounded(bar(kPFull + u % 2), static_cast<uint32_t>((u / 2) & 1))" in src
    assert "kNumBars = 17," in src


@pytest.mark.parametrize("D,S", list(itertools.product((64, 128), (16, 32))))
def test_shared_memory_and_tmem_bounds(D: int, S: int) -> None:
    c = cfg(D, S)
    assert c["launch"] <= 227 * 1024
    # exactly two CTAs per SM by shared memory, and their TMEM fits the SM's 512 columns (so
    # tcgen05.alloc never has to wait for another CTA's columns)
    ctas = SM_SMEM // (c["launch"] + 1024)
    assert ctas == 2
    assert ctas * TMEM_COLS <= TMEM_PER_SM
    q0 = 0
    k0 = q0 + c["q"]
    v0 = k0 + K_SLOTS * c["kv"]
    bars0 = v0 + V_SLOTS * c["kv"]
    assert bars0 + 17 * 8 + 4 <= c["layout"]  # 17 mbarriers + the TMEM address
    for off in (k0, v0, bars0, c["kv"]):
        assert off % 1024 == 0
    # the layout fits after aligning any 256-byte aligned base up to 1024 bytes
    assert all((-base) % 1024 + c["layout"] <= c["smem"] for base in range(0, 4096, 256))
    # Q by TMA: box b (64 columns x 128 rows of 128 B) at b * 16 KB, 1024-byte aligned, and
    # the expect-tx count (the whole tile) equals what the boxes deliver
    for b in range(c["boxes"]):
        assert (b * c["q_box"]) % 1024 == 0 and b * c["q_box"] + KM * 128 <= c["q"]
    assert c["boxes"] * 64 * KM * 2 == c["q"]
    # the epilogue's O writes into the Q tile's space: rows < 128, 16-byte chunks < D / 8,
    # and each warp's TMA store source (32 rows of box b) stays inside the tile
    assert max(sw128_off(r, ch) for r in range(KM) for ch in range(D // 8)) + 16 <= c["q"]
    for w in range(4):
        for b in range(c["boxes"]):
            src = b * c["q_box"] + w * 32 * 128
            assert src % 1024 == 0 and src + 32 * 128 <= c["q"]
            # the rows a warp's threads write are exactly its store box's rows
            rows = {(sw128_off(r, 8 * b) - b * c["q_box"]) // 128 for r in range(32 * w, 32 * w + 32)}
            assert rows == set(range(32 * w, 32 * w + 32))
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
    # TMEM: S double-buffered in [0, 64) and [64, 128), O in [128, 128 + D); P(t) in the
    # first KN / 2 columns of buffer t % 2 (pairs), the P V MMAs' A operands 8 columns each
    assert 2 * KN <= O_COL and O_COL + D <= TMEM_COLS
    for sb in range(2):
        p_cols = range(KN * sb, KN * sb + KN // 2)
        a_cols = {KN * sb + 8 * kk + c for kk in range(KN // 16) for c in range(8)}
        assert a_cols == set(p_cols) and max(p_cols) < KN * (sb + 1)


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
        hkv = 3
        seen = set()
        for lin in range(n_qblocks * hkv):            # 1-D grid, KV head fastest
            h, qi = lin % hkv, lin // hkv
            qb = n_qblocks - 1 - qi if causal else qi  # heaviest blocks first when causal
            assert 0 <= qb < n_qblocks and (qb, h) not in seen
            seen.add((qb, h))
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
            # Q box (64 x G x T) starts inside the tensor; each warp's output box
            # (64 x G x 32 / G) holds rows r = 32 w .. 32 w + 31, i.e. tokens
            # t0 + 32 w / G ...; a box that starts at or past q_len is not issued
            assert t0 < q_len
            for w in range(4):
                w_tok = t0 + w * (32 // G)
                assert [t0 + r // G for r in range(32 * w, 32 * w + 32)] == [
                    w_tok + i // G for i in range(32)]
            # a row's visible keys never exceed what the CTA loaded
            for r in range(KM):
                tok = t0 + r // G
                lim = min(kv_len, q_start + tok + 1) if causal else kv_len
                if tok < q_len:
                    assert lim <= kv_hi


class _Barrier:
    """An mbarrier: `count` arrivals complete the current phase; wait(parity) passes once
    the phase with that parity has completed (a fresh barrier passes parity 1)."""

    def __init__(self, count: int) -> None:
        self.count, self.arrived, self.phase = count, 0, 0

    def arrive(self) -> None:
        self.arrived += 1
        assert self.arrived <= self.count
        if self.arrived == self.count:
            self.arrived, self.phase = 0, self.phase + 1

    def passed(self, parity: int) -> bool:
        return (self.phase & 1) != parity


def _simulate(n_tiles: int, seed: int) -> None:  # noqa: C901
    """The kernel's three roles (load warp, MMA thread, 4 softmax warps) as coroutines over
    mbarriers, with TMA loads and MMAs completing asynchronously in random order. Checks
    that every role finishes (no deadlock) and that no buffer is overwritten before its
    previous reader or writer has finished."""
    import random

    rnd = random.Random(seed)
    B = {name: _Barrier(4 if name.startswith(("SEmpty", "PFull")) else 1) for name in
         ["KFull0", "KFull1", "KEmpty0", "KEmpty1", "VFull0", "VFull1", "VEmpty0", "VEmpty1",
          "SFull0", "SFull1", "SEmpty0", "SEmpty1", "PFull0", "PFull1", "OFree", "Drain",
          "QFull"]}
    done = {"K": set(), "V": set(), "S": set(), "PV": set(), "Q": set()}
    s_reads = [0] * max(n_tiles, 1)   # softmax warps that have read S(t)
    p_writes = [0] * max(n_tiles, 1)  # softmax warps that have written their rows of P(t)
    pending = []          # async completions: (kind, tile, barriers to arrive on)
    issued_mma = []       # MMAs in issue order (they complete in order)

    def load_warp():
        if n_tiles > 0:
            pending.append(("Q", 0, ["QFull"]))
        for t in range(n_tiles):
            sl = t % 2
            for kind in ("K", "V"):
                empty = ("KEmpty" if kind == "K" else "VEmpty") + str(sl)
                while not B[empty].passed(((t // 2) & 1) ^ 1):
                    yield
                # the slot's previous tile has been read by a completed MMA
                if t >= 2:
                    assert (t - 2) in (done["S"] if kind == "K" else done["PV"]), (kind, t)
                pending.append((kind, t, [("KFull" if kind == "K" else "VFull") + str(sl)]))

    def mma_thread():
        def pv(u):
            while not (B["PFull" + str(u % 2)].passed((u // 2) & 1) and
                       B["VFull" + str(u % 2)].passed((u // 2) & 1)):
                yield
            assert p_writes[u] == 4 and u in done["V"]
            issued_mma.append(("PV", u, ["OFree", "VEmpty" + str(u % 2)]))

        if n_tiles > 0:
            while not B["QFull"].passed(0):
                yield
            assert 0 in done["Q"]
        for t in range(n_tiles):
            sl = t % 2
            while not (B["KFull" + str(sl)].passed((t // 2) & 1) and
                       B["SEmpty" + str(sl)].passed(((t // 2) & 1) ^ 1)):
                yield
            assert t in done["K"]
            if t >= 2:
                assert s_reads[t - 2] == 4  # S buffer sl was read by every warp before reuse
            issued_mma.append(("S", t, ["SFull" + str(sl), "KEmpty" + str(sl)]))
            if t >= 1:
                yield from pv(t - 1)
        if n_tiles > 0:
            yield from pv(n_tiles - 1)
        issued_mma.append(("Drain", -1, ["Drain"]))

    def softmax_warp(w):
        for j in range(n_tiles):
            while not B["SFull" + str(j % 2)].passed((j // 2) & 1):
                yield
            assert j in done["S"]
            yield  # reading S
            s_reads[j] += 1
            B["SEmpty" + str(j % 2)].arrive()
            # P(j) goes over S(j) in TMEM buffer j % 2: the P V that read P(j - 2) there
            # has completed (S(j) was written after it, in issue order)
            assert j < 2 or (j - 2) in done["PV"]
            if j > 0 and rnd.random() < 0.3:  # a row's maximum moved: rescale O
                while not B["OFree"].passed((j - 1) & 1):
                    yield
                assert (j - 1) in done["PV"]  # O free
            if j == n_tiles - 1:
                while not B["VFull" + str(j % 2)].passed((j // 2) & 1):
                    yield
                assert j in done["V"]
            p_writes[j] += 1
            B["PFull" + str(j % 2)].arrive()
        if n_tiles > 0:
            while not B["Drain"].passed(0):
                yield
            assert (n_tiles - 1) in done["PV"]
            # the epilogue writes O into the Q tile's space: Q has landed and no S = Q K^T
            # is still reading it
            assert 0 in done["Q"] and done["S"] == set(range(n_tiles))

    roles = [load_warp(), mma_thread()] + [softmax_warp(w) for w in range(4)]
    alive = list(roles)
    steps = 0
    while alive or pending or issued_mma:
        steps += 1
        assert steps < 200000, "no progress: deadlock"
        choices = list(alive)
        if pending:
            choices.append("load")
        if issued_mma:
            choices.append("mma")
        c = rnd.choice(choices)
        if c == "load":
            kind, t, bars = pending.pop(rnd.randrange(len(pending)))
            done[kind].add(t)
            for b in bars:
                B[b].arrive()
        elif c == "mma":
            kind, t, bars = issued_mma.pop(0)  # tcgen05 MMAs complete in issue order
            if kind != "Drain":
                done[kind].add(t)
            for b in bars:
                B[b].arrive()
        else:
            try:
                next(c)
            except StopIteration:
                alive.remove(c)
    assert done["PV"] == set(range(n_tiles))


@pytest.mark.parametrize("n_tiles", [0, 1, 2, 3, 7, 16])
def test_warp_specialized_protocol_has_no_deadlock_or_early_reuse(n_tiles: int) -> None:
    for seed in range(40):
        _simulate(n_tiles, seed)
