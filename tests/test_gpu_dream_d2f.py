"""Dream on the D2F graph: the exact-K/V block_threshold device session on the GPU, through the C ABI.

The SDK's shipped CUDA profile (python/src/edllm/backends/cuda_profile.py:96-119) runs Dream with a
d2f_hybrid graph (prompt bidirectional, blocks of 8 counted from the prompt), exact K/V reuse
(exact_kv = d2f_hybrid and block_threshold, python/src/edllm/model.py:991) and the block-threshold
policy, with the Dream logits convention (position p scored from row p - 1; the row before a frozen
boundary — the shift feeder — is forwarded again, as D2FForwardPlan does,
python/src/edllm/backends/mlx_state_cache.py:557-603). Checked here:

* propose_device under the SDK's frozen / window rule agrees with the cache-free oracle forward of
  the same window (MLX contract, d2f mask with the prompt origin, shifted rows);
* the device-resident block_threshold decode equals the host-driven loop (device proposals, oracle
  BlockThresholdCommit, device commits) step for step, with threshold multi-commits exercised.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import forward as ofwd  # noqa: E402
from oracle import policy as opol  # noqa: E402
from oracle import selector as osel  # noqa: E402
from oracle.numerics import synth_weights  # noqa: E402

pytestmark = pytest.mark.gpu

DREAM_D2F = dict(layer_count=2, hidden_size=256, attention_heads=4, num_kv_heads=2, head_dim=128,
                 intermediate_size=512, vocab_size=4096, qk_norm=False, qkv_bias=True, tied_lm_head=False,
                 logits_shift=True, mask_origin="prompt", rms_norm_eps=1e-6, rope_theta=1e6, mask_token_id=4000,
                 eos_token_id=4001, block_size=8)
STD = dict(linear_std=0.05, embed_std=0.5, bias_std=0.02)
SEED = 13
BS = 8


@pytest.fixture(scope="module")
def rt():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import Runtime, build

    build.build()
    r = Runtime(model_config=DREAM_D2F, max_seq=256, max_prefill_rows=128)
    r.init_synthetic(SEED, **STD)
    yield r
    r.close()


@pytest.fixture(scope="module")
def weights():
    return synth_weights(DREAM_D2F, SEED, **STD)


def _prompt(n, seed, vocab=4000):
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, size=n)]


def _sdk_window(frontier, origin, canvas_len):
    """The SDK's proposal geometry for a non-BD3 d2f policy (device_runtime.py _run_device_state)."""
    block = (min(frontier) - origin) // BS
    frozen = origin + block * BS
    return frozen, min(canvas_len, frozen + BS)


def test_propose_matches_oracle_forward(rt, weights):
    mask = DREAM_D2F["mask_token_id"]
    P = 21  # not a multiple of the block: blocks are counted from the prompt
    x = _prompt(P, 4) + [mask] * 24
    with rt.session({"decode_strategy": "block_threshold", "attention_mask_kind": "d2f_hybrid", "block_size": BS}) as s:
        s.start_device(x, prompt_len=P, block_size=BS, mask_token_id=mask, exact_kv=True, steps=24)
        for lo in (P, P + BS, P + 2 * BS):
            # round 1 of the block: every row masked; round 2: the last half, after committing the first
            for rnd, frontier in enumerate((list(range(lo, lo + BS)), list(range(lo + BS // 2, lo + BS)))):
                frozen, end = _sdk_window(frontier, P, len(x))
                scores, tokens, fwd = s.propose_device(frontier, window_end=end, frozen_prefix=frozen)
                # exact reuse: the first forward prefills the prompt, then forwards the block and the
                # shift feeder row (the last prompt row) again; a block's first round recomputes the
                # finished block before it; a later round forwards the block and the feeder row
                if lo == P and rnd == 0:
                    assert fwd == end + 1
                elif rnd == 0:
                    assert fwd == end - frozen + BS
                else:
                    assert fwd == end - frozen + 1
                logits = ofwd.forward_mlx(weights, DREAM_D2F, x[:end], prompt_len=P, block_size=BS,
                                          output_rows=ofwd.dream_raw_rows(frontier))
                want_conf, want_tok = osel.max_prob_rows(osel.exclude_mask_token(logits, mask))
                scale = float(np.abs(logits).max())
                top2 = np.sort(logits, axis=1)[:, -2:]
                clear = (top2[:, 1] - top2[:, 0]) > 0.02 * scale
                assert np.all(np.asarray(tokens)[clear] == np.asarray(want_tok)[clear])
                np.testing.assert_allclose(scores, want_conf, rtol=0.1)
                # commit half the block (round 1) or the rest (round 2) with the device's tokens
                take = BS // 2 if rnd == 0 else len(frontier)
                s.commit_device(frontier[:take], tokens[:take])
                for p, t in zip(frontier[:take], tokens[:take]):
                    x[p] = t


def test_device_loop_equals_host_loop(rt):
    mask, eos = DREAM_D2F["mask_token_id"], DREAM_D2F["eos_token_id"]
    P, gen, steps, tau = 19, 40, 40, 0.9
    prompt = _prompt(P, 9)
    cfg = {"decode_strategy": "block_threshold", "attention_mask_kind": "d2f_hybrid", "block_size": BS}
    with rt.session(cfg) as s:
        dev = s.generate(prompt, max_tokens=gen, steps=steps, block_size=BS, confidence_threshold=tau,
                         mask_origin="prompt", trace_steps=64)
    with rt.session(cfg) as s:
        x = list(prompt) + [mask] * gen
        s.start_device(x, prompt_len=P, block_size=BS, mask_token_id=mask, exact_kv=True, steps=steps)
        c = opol.Canvas(list(x), P, mask, eos)
        pol = opol.BlockThreshold(block_size=BS, threshold=tau)
        host = []
        for step in range(steps):
            plan = pol.plan(c, step)
            if plan.action == "stop":
                break
            frozen, end = _sdk_window(plan.frontier, P, len(x))
            sc, tok, _ = s.propose_device(plan.frontier, window_end=end, frozen_prefix=frozen)
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
    # the threshold branch committed several rows in some round, and MASK was never proposed
    assert any(len(rows) > 1 for *_, rows in host)
    assert all(mask not in tok for _, tok, _, _ in host)
