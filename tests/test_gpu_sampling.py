"""Temperature sampling on the GPU, through the C ABI:

* drt_selector_sample reproduces the reference's own draws (golden vectors made by
  _sampled_max_prob_confidence, python/src/edllm/backends/diffusion_runtime.py:234-253): tokens
  equal wherever the row is certified (no DRT_TIE_NEAR), confidences within rtol 1e-12;
* a session's sampled propose_device equals the oracle's draw over the session's own window
  logits (same seed, forward index and positions);
* the device-resident BD3 decode at temperature > 0 equals the host-driven loop (device propose,
  oracle policy, device commit) step for step.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import policy as opol  # noqa: E402
from oracle import selector as osel  # noqa: E402

pytestmark = pytest.mark.gpu

SMALL = dict(layer_count=2, hidden_size=256, attention_heads=4, num_kv_heads=2, head_dim=128,
             intermediate_size=512, vocab_size=4096, qk_norm=True, qkv_bias=False, tied_lm_head=True,
             rms_norm_eps=1e-6, rope_theta=1e6, mask_token_id=4000, eos_token_id=4001, block_size=32)
STD = dict(linear_std=0.05, embed_std=0.5)
# An untied lm_head: the masked rows then predict varied tokens (a tied head at this embedding scale
# predicts MASK itself at every masked row, whatever the temperature).
UNTIED = dict(SMALL, tied_lm_head=False)


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import build

    build.build()
    return torch.device("cuda:0")


@pytest.fixture(scope="module")
def rt(dev):
    from diffusorrt_b200 import Runtime

    r = Runtime(model_config=UNTIED, max_seq=512, max_prefill_rows=256)
    r.init_synthetic(3, **STD)
    yield r
    r.close()


@pytest.mark.parametrize("name", ["small", "wide", "sharp"])
@pytest.mark.parametrize("tag", ["a", "b"])
def test_selector_sample_matches_reference_draws(dev, golden_dir, name, tag):
    from diffusorrt_b200 import kernels

    g = np.load(golden_dir / "selector.npz")
    logits = g[f"{name}_logits"]
    temp, _, fwd = (float(v) for v in g[f"{name}_sample_{tag}_args"])
    seed = int(g[f"{name}_sample_{tag}_seed"][0])
    pos = torch.tensor(g[f"{name}_sample_pos"].astype(np.int32), device=dev)
    x = torch.from_numpy(logits).to(dev)
    conf, tok, tie = kernels.select_sample(x, pos, temperature=temp, seed=seed, forward=int(fwd))
    torch.cuda.synchronize()
    conf, tok, tie = conf.cpu().numpy(), tok.cpu().numpy(), tie.cpu().numpy()
    want_tok = g[f"{name}_sample_{tag}_tok"]
    ok = tie == 0
    assert ok.mean() >= 0.5, tie
    np.testing.assert_array_equal(tok[ok], want_tok[ok])
    np.testing.assert_allclose(conf[ok], g[f"{name}_sample_{tag}_conf"][ok], rtol=1e-12, atol=0)
    # the oracle's margin agrees with the device's flag: unflagged rows are clear of the bound
    _, otok, gaps = osel.sampled_max_prob_rows(logits, temperature=temp, seed=seed, forward=int(fwd),
                                               positions=list(g[f"{name}_sample_pos"]))
    assert np.all(gaps[ok] > 0)


def test_selector_sample_wide_rows_against_oracle(dev):
    """Many rows at the Qwen3 vocabulary, gathered, with a forward index past the first."""
    from diffusorrt_b200 import kernels

    rng = np.random.default_rng(8)
    logits = rng.normal(0.0, 2.0, size=(40, 151936)).astype(np.float32)
    rows = np.asarray([3, 0, 39, 17, 17, 8], dtype=np.int32)
    positions = rng.integers(0, 4608, size=len(rows)).astype(np.int32)
    x = torch.from_numpy(logits).to(dev)
    conf, tok, tie = kernels.select_sample(x, torch.from_numpy(positions).to(dev), temperature=0.9, seed=77, forward=5,
                                           row_index=torch.from_numpy(rows).to(dev))
    torch.cuda.synchronize()
    want_conf, want_tok, gaps = osel.sampled_max_prob_rows(logits[rows], temperature=0.9, seed=77, forward=5,
                                                           positions=list(positions))
    ok = tie.cpu().numpy() == 0
    assert ok.all(), gaps
    assert tok.cpu().tolist() == want_tok
    np.testing.assert_allclose(conf.cpu().numpy(), want_conf, rtol=1e-12, atol=0)


def _prompt(n, seed, vocab=4000):
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, size=n)]


def _window_logits(s, ids, scope):
    res = s.execute_window(ids, scope, mask_geometry=(0, 32))
    return np.frombuffer(res.logits, dtype="<f4").reshape(res.n_rows, res.n_vocab)


def test_sampled_propose_matches_oracle_draw(rt):
    """The session's draw over its own logits is the reference draw (forward index = proposes since
    start_device, keyed by the frontier positions)."""
    mask = SMALL["mask_token_id"]
    prompt = _prompt(64, 31)
    x = prompt + [mask] * 32
    frontier = list(range(64, 96))
    with rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
        s.start_device(x, prompt_len=0, block_size=32, mask_token_id=mask, exact_kv=True, steps=32,
                       temperature=1.3, seed=424242)
        draws = [s.propose_device(frontier, window_end=96, frozen_prefix=64) for _ in range(3)]
        logits = _window_logits(s, x, frontier)
    # The proposals run the decode kernels, the window the prefill kernels: their logits differ within
    # the bf16 forward tolerance, which bounds how far a key or a log-probability can move.
    from bf16_tolerance import MAX_FACTOR, U_BF16

    err = MAX_FACTOR * U_BF16 * float(np.sqrt(np.mean(np.square(logits))))
    for fwd, (scores, tokens, _) in enumerate(draws):
        want_conf, want_tok, gaps = osel.sampled_max_prob_rows(logits, temperature=1.3, seed=424242, forward=fwd,
                                                               positions=frontier)
        # rows whose two best keys are within twice the logit error may draw differently
        clear = gaps > 1.3 * 2.0 ** -16 + 2 * err
        assert clear.mean() >= 0.5
        assert [t for t, c in zip(tokens, clear) if c] == [t for t, c in zip(want_tok, clear) if c], fwd
        # log p of the drawn token moves by at most the error of its logit and of the row's log-sum-exp
        assert np.all(np.abs(np.log(np.asarray(scores)[clear]) - np.log(want_conf[clear])) <= 2 * err), fwd
    # each forward index draws differently
    assert draws[0][1] != draws[1][1]


def test_sampled_device_loop_equals_host_loop(rt):
    prompt = _prompt(64, 12)
    mask, eos = SMALL["mask_token_id"], SMALL["eos_token_id"]
    gen, steps, T, seed = 64, 32, 0.8, 99
    with rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
        dev = s.generate(prompt, max_tokens=gen, steps=steps, block_size=32, temperature=T, seed=seed, trace_steps=64)
    with rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
        x = list(prompt) + [mask] * gen
        s.start_device(x, prompt_len=0, block_size=32, mask_token_id=mask, exact_kv=True, steps=steps,
                       temperature=T, seed=seed)
        c = opol.Canvas(list(x), len(prompt), mask, eos)
        pol = opol.BD3FixedQuota(block_size=32, steps=steps, prompt_len=len(prompt), gen_len=gen)
        host = []
        for step in range(pol.iteration_limit):
            plan = pol.plan(c, step)
            if plan.action == "stop":
                break
            if plan.action == "skip":
                continue
            frozen = (min(plan.frontier) // 32) * 32
            sc, tok, _ = s.propose_device(plan.frontier, window_end=plan.window_end, frozen_prefix=frozen)
            rows = pol.select(np.asarray(sc))
            pos = [plan.frontier[r] for r in rows]
            s.commit_device(pos, [tok[r] for r in rows])
            for p, r in zip(pos, rows):
                c.x[p] = tok[r]
            host.append((list(plan.frontier), list(tok), list(sc), sorted(rows)))
    assert dev["forward_count"] == len(host)
    assert dev["x"] == c.x
    for i, (tr, (frontier, tok, sc, rows)) in enumerate(zip(dev["trace"], host)):
        assert tr["frontier"] == frontier, i
        assert tr["tokens"] == tok, i
        np.testing.assert_array_equal(np.asarray(tr["scores"]), np.asarray(sc))
        assert tr["chosen"] == rows, i
    # a different seed draws a different decode
    with rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
        other = s.generate(prompt, max_tokens=gen, steps=steps, block_size=32, temperature=T, seed=seed + 1)
    assert other["x"] != dev["x"]


def test_threshold_policy_refuses_a_temperature(rt):
    mask = SMALL["mask_token_id"]
    with rt.session({"decode_strategy": "block_threshold", "block_size": 32}) as s:
        with pytest.raises(ValueError):
            s.start_device(_prompt(32, 1) + [mask] * 32, prompt_len=32, block_size=32, mask_token_id=mask,
                           exact_kv=True, steps=8, temperature=0.5)
        with pytest.raises(ValueError):
            s.generate(_prompt(32, 1), max_tokens=32, steps=8, temperature=0.5)
