"""Device-session parity on the GPU, through the C ABI (diffusorrt_b200.runtime):

* the seeded synthetic weights on the device equal the CPU restatement bit for bit;
* execute_window logits match the CPU oracle of the reference MLX forward within a bf16
  tolerance (d2f_hybrid block-causal mask, QK-norm, GQA, RoPE);
* propose_device (prefix K/V cache) agrees with a cache-free window forward;
* the device-resident decode loop equals the host-driven loop over the same session calls,
  step for step, for BD3 fixed-quota and block-threshold;
* the whole decode agrees with the CPU oracle along the device trajectory within the stated tolerance.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import forward as ofwd  # noqa: E402
from oracle import policy as opol  # noqa: E402
from oracle import selector as osel  # noqa: E402
from oracle.numerics import synth_weights  # noqa: E402

from bf16_tolerance import assert_logits_close  # noqa: E402

pytestmark = pytest.mark.gpu

SMALL = dict(layer_count=2, hidden_size=256, attention_heads=4, num_kv_heads=2, head_dim=128,
             intermediate_size=512, vocab_size=4096, qk_norm=True, qkv_bias=False, tied_lm_head=True,
             rms_norm_eps=1e-6, rope_theta=1e6, mask_token_id=4000, eos_token_id=4001, block_size=32)
STD = dict(linear_std=0.05, embed_std=0.5)
SEED = 3


@pytest.fixture(scope="module")
def rt():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import Runtime, build

    build.build()
    r = Runtime(model_config=SMALL, max_seq=512, max_prefill_rows=256)
    r.init_synthetic(SEED, **STD)
    yield r
    r.close()


@pytest.fixture(scope="module")
def weights():
    return synth_weights(SMALL, SEED, **STD)


def _prompt(n, seed, vocab=4000):
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, size=n)]


def test_synthetic_weights_match_cpu_generator(rt, weights):
    H = SMALL["hidden_size"]
    for key, shape in [("model.embed_tokens.weight", (4096, H)), ("model.layers.1.self_attn.k_proj.weight", (256, H)),
                       ("model.layers.0.mlp.up_proj.weight", (512, H)), ("model.layers.1.mlp.down_proj.weight", (H, 512)),
                       ("model.layers.0.self_attn.o_proj.weight", (H, 512))]:
        np.testing.assert_array_equal(rt.get_tensor(key, shape), weights[key])


def _window_logits(s, ids, scope):
    res = s.execute_window(ids, scope, mask_geometry=(0, 32))
    return np.frombuffer(res.logits, dtype="<f4").reshape(res.n_rows, res.n_vocab)


def test_execute_window_matches_oracle(rt, weights):
    ids = _prompt(96, 1)
    for p in (70, 71, 80, 90, 95):
        ids[p] = SMALL["mask_token_id"]
    scope = [64, 70, 71, 80, 90, 95, 3, 33]
    with rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
        got = _window_logits(s, ids, scope)
    want = ofwd.forward_mlx(weights, SMALL, ids, prompt_len=0, block_size=32, output_rows=scope)
    assert_logits_close(got, want)


def test_execute_window_long_prefix_chunks(rt, weights):
    """A window longer than one prefill chunk (256 rows) and not a multiple of the tile."""
    ids = _prompt(301, 2)
    scope = [0, 255, 256, 288, 300]
    with rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
        got = _window_logits(s, ids, scope)
    want = ofwd.forward_mlx(weights, SMALL, ids, prompt_len=0, block_size=32, output_rows=scope)
    assert_logits_close(got, want)


def test_propose_agrees_with_window_forward(rt):
    prompt = _prompt(64, 3)
    mask = SMALL["mask_token_id"]
    x = prompt + [mask] * 64
    with rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
        s.start_device(x, prompt_len=0, block_size=32, mask_token_id=mask, exact_kv=True, steps=64)
        frontier = list(range(64, 96))
        scores, tokens, fwd = s.propose_device(frontier, window_end=96, frozen_prefix=64)
        assert fwd == 96
        ref = _window_logits(s, x[:96], frontier)
    want_conf, want_tok = osel.max_prob_rows(ref)
    agree = np.mean(np.asarray(tokens) == np.asarray(want_tok))
    assert agree >= 0.9
    np.testing.assert_allclose(scores, want_conf, rtol=0.05)


@pytest.mark.parametrize("max_seq,n_prefix", [(328, 296), (2048, 1952), (6144, 6048)])
def test_long_prefix_decode_attention(max_seq, n_prefix):
    """The decode step's split-KV attention over a long cached prefix (prefilled by the first
    propose, then the 32 active rows forwarded as a decode step) agrees with the cache-free window
    forward: at 328 the keys end in a partial sixth sub-tile (two splits), at 2048 the splits of a
    KV head (7) merge inside one thread-block cluster, at 6144 (20 splits, more than a cluster
    holds) through the separate merge kernel."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import Runtime

    r = Runtime(model_config=SMALL, max_seq=max_seq, max_prefill_rows=256)
    try:
        r.init_synthetic(SEED, **STD)
        prompt = _prompt(n_prefix, max_seq)
        mask = SMALL["mask_token_id"]
        x = prompt + [mask] * 32
        with r.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
            s.start_device(x, prompt_len=0, block_size=32, mask_token_id=mask, exact_kv=True, steps=32)
            frontier = list(range(n_prefix, n_prefix + 32))
            scores, tokens, fwd = s.propose_device(frontier, window_end=n_prefix + 32, frozen_prefix=n_prefix)
            assert fwd == n_prefix + 32
            ref = _window_logits(s, x, frontier)
    finally:
        r.close()
    want_conf, want_tok = osel.max_prob_rows(ref)
    assert np.mean(np.asarray(tokens) == np.asarray(want_tok)) >= 0.9
    np.testing.assert_allclose(scores, want_conf, rtol=0.05)


def test_four_query_heads_per_kv_head_64_row_forward():
    """GQA 4:1 (8 query heads on 2 KV heads): after a block is committed, the next proposal forwards
    64 rows (the finished block again, then the new block), which with 4 query heads per KV head
    exceeds the decode attention kernel's 128 UMMA rows; the session takes the general attention
    kernel and the scores agree with the cache-free window forward."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import Runtime

    cfg = dict(SMALL, attention_heads=8, num_kv_heads=2)
    r = Runtime(model_config=cfg, max_seq=256, max_prefill_rows=128)
    try:
        r.init_synthetic(SEED, **STD)
        mask = cfg["mask_token_id"]
        x = _prompt(64, 8) + [mask] * 64
        with r.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
            s.start_device(x, prompt_len=0, block_size=32, mask_token_id=mask, exact_kv=True, steps=4)
            first = list(range(64, 96))
            _, tok, _ = s.propose_device(first, window_end=96, frozen_prefix=64)
            s.commit_device(first, tok)
            for p, t in zip(first, tok):
                x[p] = t
            frontier = list(range(96, 128))
            scores, tokens, fwd = s.propose_device(frontier, window_end=128, frozen_prefix=96)
            assert fwd == 64
            ref = _window_logits(s, x, frontier)
    finally:
        r.close()
    want_conf, want_tok = osel.max_prob_rows(ref)
    assert np.mean(np.asarray(tokens) == np.asarray(want_tok)) >= 0.9
    np.testing.assert_allclose(scores, want_conf, rtol=0.05)


def test_large_vocab_head_matches_oracle():
    """A vocabulary of 320 weight tiles (more than two per SM) takes the persistent lm_head kernel:
    one CTA per SM over a contiguous run of tiles, activation tile loaded once, TMEM accumulator
    double-buffered. Its logits match the CPU oracle at both MMA widths (20 and 48 rows)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import Runtime

    cfg = dict(SMALL, vocab_size=40960, mask_token_id=40000, eos_token_id=40001)
    r = Runtime(model_config=cfg, max_seq=256, max_prefill_rows=256)
    try:
        r.init_synthetic(SEED, **STD)
        weights = synth_weights(cfg, SEED, **STD)
        ids = _prompt(96, 5, vocab=40000)
        with r.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
            for scope in (list(range(70, 90)), list(range(0, 96, 2))):
                got = _window_logits(s, ids, scope)
                want = ofwd.forward_mlx(weights, cfg, ids, prompt_len=0, block_size=32, output_rows=scope)
                assert_logits_close(got, want)
    finally:
        r.close()


def _host_loop(s, prompt, *, strategy, gen, steps, bs, tau=0.9, cap=0):
    """The reference run_decode_loop over propose_device / commit_device (oracle policy)."""
    mask, eos = SMALL["mask_token_id"], SMALL["eos_token_id"]
    x = list(prompt) + [mask] * gen
    s.start_device(x, prompt_len=0, block_size=bs, mask_token_id=mask, exact_kv=True, steps=steps)
    c = opol.Canvas(x, len(prompt), mask, eos)
    if strategy == "bd3_fixed_quota":
        pol = opol.BD3FixedQuota(block_size=bs, steps=steps, prompt_len=len(prompt), gen_len=gen)
        limit = pol.iteration_limit
    else:
        pol = opol.BlockThreshold(block_size=bs, threshold=tau, rounds_cap=cap)
        limit = steps
    trace = []

    def score(canvas, frontier, window_end, step):
        frozen = (min(frontier) // bs) * bs
        sc, tok, _ = s.propose_device(frontier, window_end=window_end, frozen_prefix=frozen)
        return np.asarray(sc), tok

    orig_select = pol.select

    def select(scores):
        rows = orig_select(scores)
        return rows

    pol.select = select
    out = opol.run_loop(c, pol, score, limit, trace=trace)
    # commit_device mirrors the host commits
    return out, trace


@pytest.mark.parametrize("strategy,gen,steps,cap", [("bd3_fixed_quota", 96, 96, 0), ("bd3_fixed_quota", 64, 16, 0),
                                                    ("block_threshold", 64, 48, 8)])
def test_device_loop_equals_host_loop(rt, strategy, gen, steps, cap):
    prompt = _prompt(64, 11)
    mask = SMALL["mask_token_id"]
    with rt.session({"decode_strategy": strategy, "block_size": 32}) as s:
        dev = s.generate(prompt, max_tokens=gen, steps=steps, block_size=32, decode_strategy=strategy,
                         confidence_threshold=0.9, rounds_per_block=cap, trace_steps=256)

    with rt.session({"decode_strategy": strategy, "block_size": 32}) as s:
        # Host-driven loop: propose on the device, select on the host (oracle), commit on the device.
        x = list(prompt) + [mask] * gen
        s.start_device(x, prompt_len=0, block_size=32, mask_token_id=mask, exact_kv=True, steps=steps)
        c = opol.Canvas(list(x), len(prompt), mask, SMALL["eos_token_id"])
        if strategy == "bd3_fixed_quota":
            pol = opol.BD3FixedQuota(block_size=32, steps=steps, prompt_len=len(prompt), gen_len=gen)
            limit = pol.iteration_limit
        else:
            pol = opol.BlockThreshold(block_size=32, threshold=0.9, rounds_cap=cap)
            limit = steps
        host_steps = []

        def score(canvas, frontier, window_end, step):
            frozen = (min(frontier) // 32) * 32
            sc, tok, _ = s.propose_device(frontier, window_end=window_end, frozen_prefix=frozen)
            host_steps.append((list(frontier), list(tok), list(sc)))
            return np.asarray(sc), tok

        commits = []
        sel = pol.select

        def select(scores):
            rows = sel(scores)
            commits.append(sorted(rows))
            return rows

        pol.select = select
        # run the loop manually so commits go to the device too
        out = None
        forwards = 0
        for step in range(limit):
            plan = pol.plan(c, step)
            if plan.action == "stop":
                break
            if plan.action == "skip":
                continue
            scores, tokens = score(c, plan.frontier, plan.window_end, step)
            forwards += 1
            rows = pol.select(scores)
            pos = [plan.frontier[r] for r in rows]
            tok = [int(tokens[r]) for r in rows]
            s.commit_device(pos, tok)
            for p, t in zip(pos, tok):
                c.x[p] = t
        out = c.finalize()

    assert dev["forward_count"] == forwards
    assert dev["x"] == c.x
    for i, (tr, (frontier, tok, sc)) in enumerate(zip(dev["trace"], host_steps)):
        assert tr["frontier"] == frontier, i
        assert tr["tokens"] == tok, i
        np.testing.assert_array_equal(np.asarray(tr["scores"]), np.asarray(sc))
        assert tr["chosen"] == commits[i], i
    assert out is not None


def test_decode_matches_cpu_oracle_along_trajectory(rt, weights):
    """Whole BD3 decode vs the CPU oracle (MLX-contract forward + reference selector and policy),
    step by step along the device's trajectory: every step's confidences, chosen rows and tokens
    are the oracle's within the stated bf16 logit tolerance (tests/decode_check.py)."""
    from decode_check import check_bd3_trajectory

    prompt = _prompt(64, 21)
    gen, steps, bs = 64, 64, 32
    with rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": bs}) as s:
        dev = s.generate(prompt, max_tokens=gen, steps=steps, block_size=bs, trace_steps=256)
    report = check_bd3_trajectory(dev, weights, SMALL, prompt, gen=gen, steps=steps, block_size=bs)
    print("toy decode", report)
    assert report["steps"] == 64
    assert report["exact_steps"] >= report["steps"] // 4, report
