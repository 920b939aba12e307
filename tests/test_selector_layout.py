"""Column layout of the selector's first pass (diffusorrt_b200/csrc/selector.cuh, sel_pass1_kernel),
restated on the CPU: value i of thread t in a chunk starting at `lo` is column
lo + ((i / 4) * 256 + t) * 4 + i % 4 (float4 groups, 256 threads, 32 values each). The layout covers
the 8192 columns of a chunk once, each thread's values ascend in i (the first-index search relies
on it), and the excluded column's owner thread ((c - lo) / 4) % 256 and slot
((c - lo) / 4 / 256) * 4 + (c - lo) % 4 hold exactly that column.
"""
from __future__ import annotations

THREADS, CHUNK = 256, 8192


def _col(lo: int, t: int, i: int) -> int:
    return lo + ((i // 4) * THREADS + t) * 4 + i % 4


def test_selector_chunk_layout():
    lo = 3 * CHUNK
    seen = set()
    for t in range(THREADS):
        cols = [_col(lo, t, i) for i in range(CHUNK // THREADS)]
        assert cols == sorted(cols)
        seen.update(cols)
    assert seen == set(range(lo, lo + CHUNK))


def test_excluded_column_owner():
    lo = 5 * CHUNK
    for c in range(lo, lo + CHUNK):
        t = ((c - lo) >> 2) & (THREADS - 1)
        slot = (((c - lo) >> 2) // THREADS) * 4 + ((c - lo) & 3)
        assert 0 <= slot < CHUNK // THREADS
        assert _col(lo, t, slot) == c
