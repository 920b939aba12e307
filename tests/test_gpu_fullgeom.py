"""Parity at the north-star geometries on the GPU, through the C ABI, against the CPU oracle:

* Qwen3-0.6B BD3LM (28 layers, hidden 1024, 16 / 8 heads, intermediate 3072, vocabulary 151936, tied
  lm_head; python/src/edllm/backends/cuda_profile.py:151-162) with the seeded N(0, 0.02^2) weights:
  window logits of a cfg0 frontier within the stated bf16 tolerance (tests/bf16_tolerance.py), and
  whole cfg0 decodes (prompt 64, 128 new tokens, 128 steps, bd3_fixed_quota k = 1) checked step by
  step along the device's trajectory (tests/decode_check.py) for two prompt seeds;
* the Dream-7B width with its GQA 7:1 head split (hidden 3584, 28 / 4 heads, intermediate 18944,
  vocabulary 152064, q/k/v bias, untied lm_head), truncated to two layers: the full-canvas window
  logits (bidirectional, Dream logits shift) within the same tolerance, and an entropy_count decode
  whose every step scores the oracle's NegEntropy(T 0.2, top-p 0.95) within tolerance.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from bf16_tolerance import MAX_FACTOR, U_BF16, assert_logits_close  # noqa: E402
from oracle import forward as ofwd  # noqa: E402
from oracle import policy as opol  # noqa: E402
from oracle import selector as osel  # noqa: E402
from oracle.numerics import synth_weights  # noqa: E402

pytestmark = pytest.mark.gpu

STD = dict(linear_std=0.02, embed_std=0.02, bias_std=0.02)


def _qwen():
    from diffusorrt_b200.config import QWEN3_06B_BD3LM

    return dict(QWEN3_06B_BD3LM)


def _prompt(n, seed):
    return [int(t) for t in np.random.default_rng(seed).integers(0, 151643, size=n)]


@pytest.fixture(scope="module")
def qwen():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import Runtime, build

    build.build()
    cfg = _qwen()
    rt = Runtime(model_config=cfg, max_seq=256, max_prefill_rows=256)
    rt.init_synthetic(0, **STD)
    yield rt, cfg, synth_weights(cfg, 0, **STD)
    rt.close()


def test_qwen3_window_logits(qwen):
    rt, cfg, w = qwen
    mask = cfg["mask_token_id"]
    ids = _prompt(64, 0) + [mask] * 32
    frontier = list(range(64, 96))
    with rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
        res = s.execute_window(ids, frontier, mask_geometry=(0, 32))
    got = np.frombuffer(res.logits, dtype="<f4").reshape(res.n_rows, res.n_vocab)
    want = ofwd.forward_mlx(w, cfg, ids, prompt_len=0, block_size=32, output_rows=frontier)
    assert_logits_close(got, want)


@pytest.mark.parametrize("seed", [0, 1])
def test_qwen3_cfg0_decode_along_trajectory(qwen, seed):
    from decode_check import check_bd3_trajectory

    rt, cfg, w = qwen
    prompt = _prompt(64, seed)
    with rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
        dev = s.generate(prompt, max_tokens=128, steps=128, block_size=32, trace_steps=128)
    assert dev["forward_count"] == 128 and dev["committed_token_count"] == 128
    report = check_bd3_trajectory(dev, w, cfg, prompt, gen=128, steps=128, block_size=32)
    print("qwen3 cfg0 decode, seed", seed, report)
    assert report["steps"] == 128, report


@pytest.fixture(scope="module")
def dream2():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import Runtime, build
    from diffusorrt_b200.config import DREAM_7B

    build.build()
    cfg = dict(DREAM_7B, layer_count=2)
    rt = Runtime(model_config=cfg, max_seq=512, max_prefill_rows=512)
    rt.init_synthetic(0, **STD)
    yield rt, cfg, synth_weights(cfg, 0, **STD)
    rt.close()


def test_dream_gqa7_window_logits(dream2):
    rt, cfg, w = dream2
    ids = _prompt(256, 5) + [cfg["mask_token_id"]] * 256
    scope = list(range(256, 512, 8)) + [0, 1, 255]
    with rt.session({"decode_strategy": "entropy_count"}) as s:
        res = s.execute_window(ids, scope)
    got = np.frombuffer(res.logits, dtype="<f4").reshape(res.n_rows, res.n_vocab)
    want = ofwd.forward_mlx(w, cfg, ids, bidirectional=True, output_rows=ofwd.dream_raw_rows(scope))
    assert_logits_close(got, want)


def test_dream_width_d2f_decode_window(dream2):
    """A Dream-width decode window on the D2F graph (prompt bidirectional, blocks of 8 from it): the
    first proposal prefills the prompt and forwards one block and the shift feeder row. Its
    down_proj (28 weight tiles, K = 18944) is a stream-K linear over every SM. The proposal's
    confidences and tokens match the oracle forward of the same window within the stated bf16
    tolerance: |log conf_dev - log conf_oracle| <= 2 E, each token's oracle logit within 2 E of its
    row's maximum (E = 48 u of the logit RMS)."""
    rt, cfg, w = dream2
    mask = cfg["mask_token_id"]
    P, BS = 256, 8
    x = _prompt(P, 9) + [mask] * 32
    frontier = list(range(P, P + BS))
    with rt.session({"decode_strategy": "block_threshold", "attention_mask_kind": "d2f_hybrid", "block_size": BS}) as s:
        s.start_device(x, prompt_len=P, block_size=BS, mask_token_id=mask, exact_kv=True, steps=4)
        scores, tokens, fwd = s.propose_device(frontier, window_end=P + BS, frozen_prefix=P)
    assert fwd == P + BS + 1
    logits = ofwd.forward_mlx(w, cfg, x[:P + BS], prompt_len=P, block_size=BS,
                              output_rows=ofwd.dream_raw_rows(frontier))
    logits = osel.exclude_mask_token(logits, mask)
    want_conf, _ = osel.max_prob_rows(logits)
    finite = logits[np.isfinite(logits)]
    E = MAX_FACTOR * U_BF16 * float(np.sqrt(np.mean(finite.astype(np.float64) ** 2)))
    assert np.all(np.abs(np.log(np.asarray(scores)) - np.log(np.asarray(want_conf))) <= 2 * E)
    rows = np.arange(len(frontier))
    assert np.all(logits[rows, np.asarray(tokens)] >= logits.max(axis=1) - 2 * E)


def test_dream_width_d2f_decode_rounds(dream2):
    """Six D2F proposals at the Dream width (three blocks of 8 after a 256-token prompt, two rounds
    each). After the first, which prefills the prompt, every proposal is a decode forward of the
    window (with the finished block before it on a block's first round) over the K/V cache: the
    decode graph is sized for 64 rows, four query tiles of 18 positions at GQA 7:1, of which the
    live rows fill one or two, each tile's keys split over a cluster. Each proposal's confidences
    and tokens match the oracle forward of the same canvas within the stated bf16 tolerance
    (|log conf_dev - log conf_oracle| <= 2 E, each token's oracle logit within 2 E of its row's
    maximum, E = 48 u of the logit RMS)."""
    rt, cfg, w = dream2
    mask = cfg["mask_token_id"]
    P, BS = 256, 8
    x = _prompt(P, 12) + [mask] * 3 * BS
    mode = {"decode_strategy": "block_threshold", "attention_mask_kind": "d2f_hybrid", "block_size": BS}
    with rt.session(mode) as s:
        s.start_device(x, prompt_len=P, block_size=BS, mask_token_id=mask, exact_kv=True, steps=8)
        for lo in (P, P + BS, P + 2 * BS):
            for rnd, frontier in enumerate((list(range(lo, lo + BS)), list(range(lo + BS // 2, lo + BS)))):
                scores, tokens, fwd = s.propose_device(frontier, window_end=lo + BS, frozen_prefix=lo)
                if lo == P and rnd == 0:
                    assert fwd == P + BS + 1
                elif rnd == 0:
                    assert fwd == 2 * BS  # the finished block is recomputed with its final tokens
                else:
                    assert fwd == BS + 1
                logits = ofwd.forward_mlx(w, cfg, x[:lo + BS], prompt_len=P, block_size=BS,
                                          output_rows=ofwd.dream_raw_rows(frontier))
                logits = osel.exclude_mask_token(logits, mask)
                want_conf, _ = osel.max_prob_rows(logits)
                finite = logits[np.isfinite(logits)]
                E = MAX_FACTOR * U_BF16 * float(np.sqrt(np.mean(finite.astype(np.float64) ** 2)))
                assert np.all(np.abs(np.log(np.asarray(scores)) - np.log(np.asarray(want_conf))) <= 2 * E), (lo, rnd)
                rows = np.arange(len(frontier))
                assert np.all(logits[rows, np.asarray(tokens)] >= logits.max(axis=1) - 2 * E), (lo, rnd)
                take = BS // 2 if rnd == 0 else len(frontier)
                s.commit_device(frontier[:take], tokens[:take])
                for q, t in zip(frontier[:take], tokens[:take]):
                    x[q] = t


def test_dream_gqa7_entropy_count_along_trajectory(dream2):
    """Every step of the device's entropy_count decode (NegEntropy T 0.2 with top-p 0.95, MASK
    excluded, top-k by the f32 entropy) against the oracle on the device's canvas: each frontier
    row's entropy within the bound the logit tolerance implies, and the committed rows and tokens
    consistent with the oracle's within it."""
    rt, cfg, w = dream2
    mask = cfg["mask_token_id"]
    T, TOP_P, steps, gen = 0.2, 0.95, 6, 64  # at most 64 masked positions: the step trace holds 64 rows
    prompt = _prompt(256, 6)
    with rt.session({"decode_strategy": "entropy_count"}) as s:
        dev = s.generate(prompt, max_tokens=gen, steps=steps, temperature=T, top_p=TOP_P, eps=1e-3,
                         trace_steps=steps)
    c = opol.Canvas(list(prompt) + [mask] * gen, len(prompt), mask, cfg["eos_token_id"])
    pol = opol.EntropyCount(eps=1e-3, steps=steps)
    traces = iter(dev["trace"])
    checked = 0
    for step in range(steps):
        plan = pol.plan(c, step)
        if plan.action == "stop":
            break
        if plan.action == "skip":
            continue
        tr = next(traces)
        assert tr["frontier"] == plan.frontier
        logits = ofwd.forward_mlx(w, cfg, c.x, bidirectional=True, output_rows=ofwd.dream_raw_rows(plan.frontier))
        E = MAX_FACTOR * U_BF16 * float(np.sqrt(np.mean(np.square(logits.astype(np.float64)))))
        x = osel.exclude_mask_token(logits, mask)
        conf, tok = osel.neg_entropy_rows(x, temperature=T, top_p=TOP_P)
        # The entropy of softmax(x / T) moves by at most 2 E / T per unit of log-probability spread;
        # the committed token's logit is within 2 E of its row's maximum.
        bound = 2 * E / T * max(1.0, float(np.max(np.abs(conf))))
        assert np.all(np.abs(np.asarray(tr["scores"]) - conf) <= bound), step
        for r in tr["chosen"]:
            assert float(x[r].max() - x[r][tr["tokens"][r]]) <= 2 * E, (step, r)
        k = len(tr["chosen"])
        others = [r for r in range(len(plan.frontier)) if r not in tr["chosen"]]
        if others:
            assert max(conf[others]) - min(conf[tr["chosen"]]) <= 2 * bound, step
        assert k == len(pol.select(conf))
        for r in tr["chosen"]:
            c.x[plan.frontier[r]] = tr["tokens"][r]
        checked += 1
    assert checked == dev["forward_count"] >= 3
