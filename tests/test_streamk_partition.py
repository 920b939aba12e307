"""Index arithmetic of the stream-K linear (diffusorrt_b200/csrc/gemm_streamk.cuh), restated on the
CPU and checked over the shapes the library launches and their edge cases.

The kernel gives CTA c of G the (weight tile, K block) iterations [total c / G, total (c + 1) / G)
and walks them tile by tile. A segment that starts inside a tile (a tail) stores its partial in
the CTA's slot and raises the CTA's flag; a segment that starts at K block 0 (a head) owns the
tile, waits for the flags of CTAs c + 1 .. c_last with
c_last = ceil((last iteration of the tile + 1) G / total) - 1, adds their partials and clears the
flags. The properties: every CTA has work, at most one tail (its first segment) and hence one
partial slot; each tile has exactly one head; the CTAs a head waits for are exactly the others that
hold iterations of its tile, each of them with a tail in that tile; every tail is consumed by
exactly one head.
"""
from __future__ import annotations

import pytest


def _segments(c: int, G: int, total: int, KB: int):
    it0, it1 = total * c // G, total * (c + 1) // G
    out = []
    it = it0
    while it < it1:
        t = it // KB
        ka = it - t * KB
        kend = min(KB, it1 - t * KB)
        out.append((t, ka, kend))
        it = t * KB + kend
    return out


def _check(tiles: int, KB: int, G: int) -> None:
    total = tiles * KB
    G = min(G, total)  # the host launches min(SMs, iterations) CTAs
    heads: dict[int, int] = {}
    tails: dict[int, list[int]] = {}
    holders: dict[int, set[int]] = {}
    for c in range(G):
        segs = _segments(c, G, total, KB)
        assert segs, (tiles, KB, G, c)
        assert sum(1 for _, ka, _ in segs if ka != 0) <= 1  # one partial slot per CTA
        for i, (t, ka, kend) in enumerate(segs):
            assert 0 <= ka < kend <= KB
            holders.setdefault(t, set()).add(c)
            if ka == 0:
                assert t not in heads
                heads[t] = c
            else:
                assert i == 0  # a tail is the CTA's first segment, finished before its head
                tails.setdefault(t, []).append(c)
    consumed = set()
    for t in range(tiles):
        assert t in heads, (tiles, KB, G, t)
        c = heads[t]
        last_it = t * KB + KB - 1
        c_last = -(-(last_it + 1) * G // total) - 1
        waited = set(range(c + 1, c_last + 1))
        assert waited == holders[t] - {c}, (tiles, KB, G, t)
        assert waited == set(tails.get(t, [])), (tiles, KB, G, t)
        assert not (waited & consumed)
        consumed |= waited
    assert consumed == {c for cs in tails.values() for c in cs}


@pytest.mark.parametrize("tiles,KB", [
    (296, 56),    # Dream-7B gate/up over a decode window (37888 rows, K 3584)
    (28, 296),    # Dream-7B down_proj (3584 rows, K 18944): each tile split over about five CTAs
    (1188, 56),   # Dream-7B lm_head (152064 rows, K 3584)
    (36, 56), (1, 1), (1, 7), (3, 1), (147, 1), (149, 3), (5, 1000),
])
@pytest.mark.parametrize("G", [1, 2, 7, 148, 296])
def test_streamk_partition(tiles, KB, G):
    _check(tiles, KB, G)


def test_streamk_partition_small_exhaustive():
    for tiles in range(1, 13):
        for KB in range(1, 13):
            for G in range(1, 40):
                _check(tiles, KB, G)
