"""Key partition of the decode attention (diffusorrt_b200/csrc/attention_decode.cuh), restated on
the CPU: the session sizes the CTAs per KV head as ceil(ceil(max_seq / 64) / kDaMaxSub) (capi.cu,
session set-up), and CTA `split` of S covers the 64-key sub-tiles
[split n_sub / S, (split + 1) n_sub / S) of the current K/V length. For every K/V length up to
max_seq the CTAs tile the keys without gaps or overlap and none gets more than kDaMaxSub sub-tiles
(the kernel records DEV_BAD_GEOMETRY instead of dropping keys if one ever did).
"""
from __future__ import annotations

import pytest

K_DA_MAX_SUB = 5


def _splits(max_seq: int) -> int:
    n_sub = (max_seq + 63) // 64
    return (n_sub + K_DA_MAX_SUB - 1) // K_DA_MAX_SUB


@pytest.mark.parametrize("max_seq", [64, 65, 256, 320, 321, 4224, 4608, 8192, 20000])
def test_decode_attention_splits_cover_every_key(max_seq):
    S = _splits(max_seq)
    for kv_len in range(1, max_seq + 1, max(1, max_seq // 997)):
        n_sub = (kv_len + 63) // 64
        covered = []
        for split in range(S):
            sub0, sub1 = split * n_sub // S, (split + 1) * n_sub // S
            assert 0 <= sub1 - sub0 <= K_DA_MAX_SUB, (max_seq, kv_len, split)
            covered.extend(range(sub0, sub1))
        assert covered == list(range(n_sub)), (max_seq, kv_len)
