"""Kernel-level parity on the GPU: the tcgen05 linear against a torch fp32 reference, and the
fused selector against the CPU oracle of the reference selector on identical f32 logits."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import selector as osel  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import build

    build.build()
    return torch.device("cuda:0")


def _bf16_round_torch(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(torch.float32)


@pytest.mark.parametrize("rows,n,K,splits", [(32, 256, 1024, 1), (64, 4096, 1024, 4), (17, 1024, 3072, 16),
                                             (100, 384, 512, 2), (64, 1024, 2048, 16)])
def test_linear_matches_fp32_reference(dev, rows, n, K, splits):
    from diffusorrt_b200 import kernels

    g = torch.Generator(device="cpu").manual_seed(rows * 31 + n + K)
    x = torch.randn(rows, K, generator=g).to(torch.bfloat16).to(dev)
    w = (torch.randn(n, K, generator=g) * 0.05).to(torch.bfloat16).to(dev)
    ref = x.float() @ w.float().t()
    raw = kernels.linear_bf16(x, w, splits=splits, round_bf16=False)
    torch.cuda.synchronize()
    # f32 accumulation in a different order: relative error ~ K * 2^-24.
    tol = 1e-5 * ref.abs().max().item() + 1e-6
    assert (raw - ref).abs().max().item() <= tol
    rounded = kernels.linear_bf16(x, w, splits=splits, round_bf16=True)
    torch.cuda.synchronize()
    expect = _bf16_round_torch(ref)
    diff = (rounded - expect).abs()
    # Two f32 values `tol` apart may round to neighbouring bf16 values (one step of 2^-7
    # relative), including near zero where the f32 accumulation error dominates the value.
    bound = 2.0 ** -7 * (expect.abs() + tol) + tol
    assert bool((diff <= bound).all())
    assert (diff > 0).float().mean().item() < 0.01


def _logits(rows, vocab, seed, scale=3.0):
    rng = np.random.default_rng(seed)
    return rng.normal(0.0, scale, size=(rows, vocab)).astype(np.float32)


@pytest.mark.parametrize("rows,vocab", [(1, 151936), (32, 151936), (5, 4096), (3, 152064), (7, 8195)])
def test_selector_max_prob_matches_oracle(dev, rows, vocab):
    from diffusorrt_b200 import kernels

    x = _logits(rows, vocab, seed=rows * 1000 + vocab)
    if rows > 2:
        x[2, 17] = x[2, vocab - 5] = x[2].max() + 1.0  # exact tie on the max: first index wins
    conf, tok = kernels.select_rows(torch.from_numpy(x).to(dev))
    torch.cuda.synchronize()
    want_conf, want_tok = osel.max_prob_rows(x)
    assert tok.cpu().tolist() == want_tok
    np.testing.assert_allclose(conf.cpu().numpy(), want_conf, rtol=1e-13, atol=0)


@pytest.mark.parametrize("temperature", [1.0, 0.2])
def test_selector_entropy_matches_oracle(dev, temperature):
    from diffusorrt_b200 import _lib, kernels

    x = _logits(16, 151936, seed=7)
    conf, tok = kernels.select_rows(torch.from_numpy(x).to(dev), mode=_lib.SELECT_NEG_ENTROPY,
                                    temperature=temperature)
    torch.cuda.synchronize()
    want_conf, want_tok = osel.neg_entropy_rows(x, temperature=temperature, top_p=None)
    assert tok.cpu().tolist() == want_tok
    got = conf.cpu().numpy().astype(np.float32)
    # The f64 sums agree to ~1e-14 relative; after the f32 cast they match to one f32 step.
    np.testing.assert_allclose(got, want_conf, rtol=2.5e-7, atol=0)


def test_selector_choices_certified(dev):
    """Top-k and threshold choices from device confidences equal the reference choices from the
    oracle confidences on every certified decision."""
    from diffusorrt_b200 import kernels

    rel = 2.0 ** -40
    checked = 0
    for seed in range(20):
        x = _logits(32, 151936, seed=100 + seed, scale=3.0 + seed * 0.5)
        conf, _ = kernels.select_rows(torch.from_numpy(x).to(dev))
        torch.cuda.synchronize()
        dconf = conf.cpu().numpy()
        oconf, _ = osel.max_prob_rows(x)
        for k in (1, 4, 8):
            got, ok = osel.topk_set_certified(dconf, k, rel)
            if ok:
                assert got == set(osel.topk_choices(oconf, k))
                checked += 1
        got, ok = osel.threshold_set_certified(dconf, 0.9, rel)
        if ok:
            assert got == set(osel.threshold_choices(oconf, 0.9))
            checked += 1
    assert checked >= 70


def test_selector_throughput_sane(dev):
    """One 32 x 151936 selector pass completes and is HBM-bound-fast (< 0.2 ms)."""
    from diffusorrt_b200 import kernels

    x = torch.randn(32, 151936, device=dev) * 3
    scratch = kernels.selector_scratch(32, 151936, dev)
    for _ in range(3):
        kernels.select_rows(x, scratch=scratch)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(20):
        kernels.select_rows(x, scratch=scratch)
    e.record()
    torch.cuda.synchronize()
    assert s.elapsed_time(e) / 20 < 0.2
