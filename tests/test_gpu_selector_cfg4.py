"""Unmask-selector microbenchmark configuration (fp32 logits [B, L, V] ~ N(0, 3^2), 50% masked
positions; max-prob and entropy confidence, top-k k in {1, 4, 8} and threshold 0.9 choices), on
the GPU through the C ABI, against the CPU oracle (the reference selector restated and pinned to
its golden vectors).

Bit-exactness contract: token ids equal; confidences equal to the oracle's within the float64
summation-order bound (max-prob) or one float32 ulp (entropy, whose reference value is cast to
float32); choice sets equal on every batch item whose decision the device certifies (tie flag 0).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import selector as osel

pytestmark = pytest.mark.gpu

V = 151936
TIE_REL = 2.0 ** -40


def _case(B: int, L: int, seed: int):
    rng = np.random.default_rng(seed)
    logits = (rng.standard_normal((B, L, V), dtype=np.float32) * np.float32(3.0)).astype(np.float32)
    mask = rng.random((B, L)) < 0.5
    for b in range(B):  # every item keeps at least one masked position
        if not mask[b].any():
            mask[b, 0] = True
    return logits, mask


def _device_rows(mask):
    B, L = mask.shape
    rows, offsets = [], [0]
    for b in range(B):
        idx = np.flatnonzero(mask[b])
        rows.extend(int(b * L + i) for i in idx)
        offsets.append(len(rows))
    return rows, offsets


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from diffusorrt_b200 import build
    build.build()
    return torch.device("cuda:0")


@pytest.mark.parametrize("mode", ["max_prob", "entropy"])
@pytest.mark.parametrize("B,L", [(1, 32), (1, 256), (8, 32), (8, 256)])
def test_selector_cfg4_matches_oracle(dev, mode, B, L):
    from diffusorrt_b200 import _lib, kernels
    logits, mask = _case(B, L, seed=11 + B * 1000 + L)
    rows, offsets = _device_rows(mask)
    flat = torch.from_numpy(logits.reshape(B * L, V)).to(dev)
    ridx = torch.tensor(rows, dtype=torch.int32, device=dev)
    off = torch.tensor(offsets, dtype=torch.int32, device=dev)
    sel = logits.reshape(B * L, V)[rows]
    if mode == "max_prob":
        conf, tok = kernels.select_gather(flat, ridx, mode=_lib.SELECT_MAX_PROB)
        want_conf, want_tok = osel.max_prob_rows(sel)
        got = conf.cpu().numpy()
        np.testing.assert_allclose(got, want_conf, rtol=1e-12, atol=0)
    else:
        conf, tok = kernels.select_gather(flat, ridx, mode=_lib.SELECT_NEG_ENTROPY, temperature=1.0)
        want_conf, want_tok = osel.neg_entropy_rows(sel, temperature=1.0, top_p=None)
        got = conf.cpu().numpy().astype(np.float32)
        ulp = np.spacing(np.abs(want_conf).astype(np.float32))
        assert np.all(np.abs(got - want_conf) <= ulp), np.max(np.abs(got - want_conf) / ulp)
    assert tok.cpu().tolist() == list(want_tok)
    want_conf = np.asarray(want_conf, dtype=np.float64)
    certified = 0
    for kind, param in [("topk", 1), ("topk", 4), ("topk", 8), ("threshold", 0.9)]:
        if kind == "topk":
            chosen, tie = kernels.select_choices(conf, off, mode=kernels.CHOICE_TOPK, k=param, tie_rel=TIE_REL)
        else:
            chosen, tie = kernels.select_choices(conf, off, mode=kernels.CHOICE_THRESHOLD, tau=param, tie_rel=TIE_REL)
        chosen = chosen.cpu().numpy()
        tie = tie.cpu().numpy()
        for b in range(B):
            lo, hi = offsets[b], offsets[b + 1]
            c = want_conf[lo:hi]
            if kind == "topk":
                want_set, ok = osel.topk_set_certified(c, param, 1e-9)
                ref_set = set(osel.topk_choices(c, param))
            else:
                want_set, ok = osel.threshold_set_certified(c, param, 1e-9)
                ref_set = set(osel.threshold_choices(c, param))
            got_set = {i for i in range(hi - lo) if chosen[lo + i]}
            if tie[b] == 0 and ok:
                assert got_set == want_set == ref_set, (kind, param, b)
                certified += 1
    # every decision is certified except where the float64 keys of two rows nearly coincide
    assert certified >= 3 * B


def test_selector_cfg4_full_size_properties(dev):
    """B = 8, L = 256 on the device alone: tokens are the first index of the row maximum, the
    max-prob confidence equals 1 / sum(exp(x - max)) evaluated in float64 by torch, and the
    top-k / threshold sets equal a direct restatement on those confidences."""
    from diffusorrt_b200 import _lib, kernels
    B, L = 8, 256
    g = torch.Generator(device=dev).manual_seed(4)
    flat = torch.randn(B * L, V, generator=g, device=dev, dtype=torch.float32) * 3.0
    mask = torch.rand(B, L, generator=g, device=dev) < 0.5
    rows = torch.nonzero(mask.reshape(-1)).reshape(-1).to(torch.int32)
    counts = mask.sum(1).cpu().tolist()
    offsets = torch.tensor(np.concatenate([[0], np.cumsum(counts)]), dtype=torch.int32, device=dev)
    conf, tok = kernels.select_gather(flat, rows, mode=_lib.SELECT_MAX_PROB)
    sel = flat[rows.long()]
    assert torch.equal(tok.long(), torch.argmax(sel, dim=1))
    x = sel.double()
    ref = 1.0 / torch.exp(x - x.max(dim=1, keepdim=True).values).sum(dim=1)
    assert torch.allclose(conf, ref, rtol=1e-12, atol=0)
    for k in (1, 4, 8):
        chosen, tie = kernels.select_choices(conf, offsets, mode=kernels.CHOICE_TOPK, k=k, tie_rel=TIE_REL)
        c = conf.cpu().numpy()
        ch = chosen.cpu().numpy()
        tie = tie.cpu().numpy()
        off = offsets.cpu().tolist()
        for b in range(B):
            lo, hi = off[b], off[b + 1]
            want, ok = osel.topk_set_certified(c[lo:hi], k, TIE_REL)
            if tie[b] == 0:
                assert {i for i in range(hi - lo) if ch[lo + i]} == want
