"""CPU check of the decode-attention kernel's work partition (index math only).

paged_decode_attn.cu cuts the flattened (request, kv head, page) stream into one
contiguous range per warp, and merges the pieces of a (request, head) segment that
cross warp boundaries with a last-arriver counter. This test restates that integer
arithmetic in Python and checks, for many ragged batches and warp counts, that:

  * every stream position is owned by exactly one warp, and every active warp owns
    at least one (the kernel divides over min(warps, positions));
  * the first/last warp formulas find the warps that actually hold a segment's ends;
  * each warp emits at most one partial with role 0 and one with role 1, and the
    slots the merging warp reads are exactly the slots the pieces were written to.
"""

from __future__ import annotations

import numpy as np
import pytest


def pieces_by_walk(npages: list[int], hkv: int, nw: int):
    """Walk every warp's range like the kernel does; return segment -> [(warp, role, complete)]."""
    poff = np.concatenate([[0], np.cumsum(npages)]).astype(np.int64)
    total = int(poff[-1]) * hkv
    segs: dict[tuple[int, int], list[tuple[int, int, bool]]] = {}
    owner = np.full(total, -1)
    nwe = min(nw, total)
    for w in range(nwe):
        lo, hi = total * w // nwe, total * (w + 1) // nwe
        pos = lo
        while pos < hi:
            b = int(np.searchsorted(poff * hkv, pos, side="right") - 1)
            n = npages[b]
            rem = pos - int(poff[b]) * hkv
            h, p = divmod(rem, n)
            seg_start = int(poff[b]) * hkv + h * n
            seg_end = seg_start + n
            piece_start = pos
            piece_end = min(seg_end, hi)
            owner[piece_start:piece_end] = np.where(owner[piece_start:piece_end] < 0, w, -2)
            complete = piece_start == seg_start and piece_end == seg_end
            role = 0 if piece_start == lo else 1
            segs.setdefault((b, h), []).append((w, role, complete))
            pos = piece_end
        assert hi > lo, "an active warp with an empty range would never arrive"
    return segs, owner, total, poff


def first_warp(s: int, nw: int, total: int) -> int:
    return ((s + 1) * nw - 1) // total


def last_warp(e: int, nw: int, total: int) -> int:
    return (e * nw - 1) // total


@pytest.mark.parametrize("seed", range(40))
def test_partition_covers_and_merges(seed: int) -> None:
    rng = np.random.default_rng(seed)
    B = int(rng.integers(1, 70))
    hkv = int(rng.choice([1, 2, 4, 8]))
    nw = int(rng.choice([1, 3, 4, 64, 592, 1184]))
    npages = [int(x) for x in rng.integers(0, 40, size=B)]
    if rng.random() < 0.3:
        npages[int(rng.integers(B))] = 600  # one long context
    segs, owner, total, poff = pieces_by_walk(npages, hkv, nw)
    if total == 0:
        return
    nw = min(nw, total)  # the kernel partitions over at most `total` warps
    assert (owner >= 0).all(), "a stream position is owned by zero or two warps"
    slots_written = set()
    for (b, h), pieces in segs.items():
        n = npages[b]
        s = int(poff[b]) * hkv + h * n
        e = s + n
        wa, wb = first_warp(s, nw, total), last_warp(e, nw, total)
        assert [p[0] for p in pieces] == list(range(wa, wb + 1))
        if len(pieces) == 1:
            assert pieces[0][2], "a single-piece segment must be complete"
            continue
        role_a = 0 if total * wa // nw == s else 1
        expect = [(wa, role_a)] + [(w, 0) for w in range(wa + 1, wb + 1)]
        assert [(p[0], p[1]) for p in pieces] == expect
        for slot in expect:
            assert slot not in slots_written, "two partials share a workspace slot"
            slots_written.add(slot)


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("G", range(1, 9))
def test_merge_lane_map_covers_every_output_once(G: int, D: int) -> None:
    # merge_pieces: lane -> (head g, columns d0 .. d0 + 4*n4), lanes with g >= G idle.
    gp = 1 if G <= 1 else 2 if G <= 2 else 4 if G <= 4 else 8
    lph = 32 // gp if (32 // gp) * 4 <= D else D // 4
    n4 = D // (4 * lph)
    assert 1 <= n4 <= D // 16
    seen = np.zeros((G, D), dtype=int)
    for lane in range(32):
        g = lane // lph
        if g >= G:
            continue
        d0 = (lane % lph) * 4 * n4
        seen[g, d0:d0 + 4 * n4] += 1
    assert (seen == 1).all()
