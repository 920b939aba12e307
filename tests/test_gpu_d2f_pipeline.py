"""The D2F block-pipeline policy on the device (D2FBlockPipelineCommit,
python/src/edllm/backends/diffusion_runtime.py:1416-1704), through the C ABI.

A window of prompt-relative blocks decodes together: fully decoded blocks freeze oldest-first, a
block joins when the last one's decoded ratio reaches tau_add, a block is fully activated when the
one before it reaches tau_act, and each step commits the rows strictly above tau_conf, or a fully
activated block's single best row. Checked here, on a BD3LM-style model (absolute attention blocks)
and on a Dream-style one (logits shift, prompt as the mask origin):

* the device-resident decode equals the host-driven loop (device proposals over the window the
  oracle policy plans, oracle selection, device commits) step for step: frontier, tokens, scores,
  chosen rows, forward count and canvas, bit for bit;
* the three commit regimes occur: forced single commits (nothing clears tau_conf), threshold
  multi-commits, and windows of several blocks;
* requests whose pipeline blocks would straddle attention blocks, and out-of-range thresholds,
  are refused.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import policy as opol  # noqa: E402

pytestmark = pytest.mark.gpu

BS = 8
QWEN_SMALL = dict(layer_count=2, hidden_size=256, attention_heads=4, num_kv_heads=2, head_dim=128,
                  intermediate_size=512, vocab_size=4096, qk_norm=True, qkv_bias=False, tied_lm_head=False,
                  rms_norm_eps=1e-6, rope_theta=1e6, mask_token_id=4000, eos_token_id=4001, block_size=BS)
DREAM_SMALL = dict(layer_count=2, hidden_size=256, attention_heads=4, num_kv_heads=2, head_dim=128,
                   intermediate_size=512, vocab_size=4096, qk_norm=False, qkv_bias=True, tied_lm_head=False,
                   logits_shift=True, mask_origin="prompt", rms_norm_eps=1e-6, rope_theta=1e6, mask_token_id=4000,
                   eos_token_id=4001, block_size=BS)
STD = dict(linear_std=0.05, embed_std=0.5, bias_std=0.02)
SESSION = {"decode_strategy": "d2f_block_pipeline", "attention_mask_kind": "d2f_hybrid", "block_size": BS}


def _prompt(n, seed, vocab=4000):
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, size=n)]


@pytest.fixture(scope="module", params=["qwen", "dream"])
def model(request):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import Runtime, build

    build.build()
    cfg = QWEN_SMALL if request.param == "qwen" else DREAM_SMALL
    r = Runtime(model_config=cfg, max_seq=256, max_prefill_rows=128)
    r.init_synthetic(17, **STD)
    yield request.param, cfg, r
    r.close()


def _geometry(kind):
    # BD3LM graph: absolute blocks, so the prompt is a whole number of blocks; Dream D2F graph:
    # blocks counted from the prompt, any prompt length
    return (64, 0) if kind == "qwen" else (21, "prompt")


def _mask_prompt_len(origin, prompt):
    """start_device's prompt_len is the d2f mask geometry's: 0 for absolute blocks."""
    return len(prompt) if origin == "prompt" else int(origin)


def _first_scores(rt, prompt, gen, origin):
    """Confidences of the first block's rows, to place tau_conf inside their range."""
    mask = rt.config["mask_token_id"]
    x = list(prompt) + [mask] * gen
    with rt.session(SESSION) as s:
        s.start_device(x, prompt_len=_mask_prompt_len(origin, prompt), block_size=BS, mask_token_id=mask,
                       exact_kv=True, steps=4)
        frontier = list(range(len(prompt), len(prompt) + BS))
        sc, _, _ = s.propose_device(frontier, window_end=len(prompt) + BS, frozen_prefix=len(prompt))
    return np.asarray(sc, dtype=np.float64)


def _host_loop(rt, prompt, gen, steps, tau, tau_add, tau_act, origin):
    mask, eos = rt.config["mask_token_id"], rt.config["eos_token_id"]
    P = len(prompt)
    x = list(prompt) + [mask] * gen
    host, windows = [], []
    with rt.session(SESSION) as s:
        s.start_device(x, prompt_len=_mask_prompt_len(origin, prompt), block_size=BS, mask_token_id=mask,
                       exact_kv=True, steps=steps)
        c = opol.Canvas(list(x), P, mask, eos)
        pol = opol.D2FPipeline(block_size=BS, threshold=tau, add_threshold=tau_add, activate_threshold=tau_act)
        for step in range(steps):
            plan = pol.plan(c, step)
            if plan.action == "stop":
                break
            windows.append((pol.frozen_end, plan.window_end))
            sc, tok, _ = s.propose_device(plan.frontier, window_end=plan.window_end, frozen_prefix=pol.frozen_end)
            rows = pol.select(np.asarray(sc))
            pos = [plan.frontier[r] for r in rows]
            s.commit_device(pos, [tok[r] for r in rows])
            for p, r in zip(pos, rows):
                c.x[p] = tok[r]
            host.append((list(plan.frontier), list(tok), list(sc), sorted(rows)))
    return c, host, windows


@pytest.mark.parametrize("regime", ["forced", "mixed", "all"])
def test_device_pipeline_equals_host_loop(model, regime):
    kind, cfg, rt = model
    P, origin = _geometry(kind)
    prompt = _prompt(P, 5 if kind == "qwen" else 6)
    gen, steps = 48, 96
    first = _first_scores(rt, prompt, gen, origin)
    tau = {"forced": 1.0, "mixed": float(np.median(first)), "all": 0.0}[regime]
    tau_add, tau_act = 0.1, 0.95
    with rt.session(SESSION) as s:
        dev = s.generate(prompt, max_tokens=gen, steps=steps, block_size=BS, decode_strategy="d2f_block_pipeline",
                         confidence_threshold=tau, add_threshold=tau_add, activate_threshold=tau_act,
                         mask_origin=origin, trace_steps=128)
    c, host, windows = _host_loop(rt, prompt, gen, steps, tau, tau_add, tau_act, origin)
    assert dev["forward_count"] == len(host)
    assert dev["x"] == c.x
    for i, (tr, (frontier, tok, sc, rows)) in enumerate(zip(dev["trace"], host)):
        assert tr["frontier"] == frontier, i
        assert tr["tokens"] == tok, i
        np.testing.assert_array_equal(np.asarray(tr["scores"]), np.asarray(sc))
        assert tr["chosen"] == rows, i
    mask = rt.config["mask_token_id"]
    assert all(mask not in tok for _, tok, _, _ in host)
    blocks_in_window = [(end - lo + BS - 1) // BS for lo, end in windows]
    if regime == "forced":
        # nothing clears tau_conf = 1: one forced row per step from the oldest block, while later
        # semi-activated blocks wait in the window
        assert all(len(rows) == 1 for *_, rows in host)
        assert max(blocks_in_window) >= 2
    elif regime == "mixed":
        assert any(len(rows) > 1 for *_, rows in host)
        assert max(blocks_in_window) >= 2
    else:
        # every masked row clears tau_conf = 0: each appended block commits whole
        assert all(len(rows) == len(frontier) for frontier, _, _, rows in host)
    assert dev["remaining_mask_count"] == 0 or dev["forward_count"] == steps


def test_pipeline_refusals(model):
    kind, cfg, rt = model
    mask = rt.config["mask_token_id"]
    with rt.session(SESSION) as s:
        if kind == "qwen":
            # absolute attention blocks: a prompt of 60 puts pipeline blocks across attention blocks
            with pytest.raises(ValueError, match="multiple of block_size"):
                s.generate(_prompt(60, 1), max_tokens=16, steps=8, block_size=BS, decode_strategy="d2f_block_pipeline",
                           mask_origin=0)
        for bad in ({"add_threshold": 0.0}, {"activate_threshold": 1.5}):
            with pytest.raises(ValueError, match="threshold"):
                s.generate(_prompt(24, 2), max_tokens=16, steps=8, block_size=BS, decode_strategy="d2f_block_pipeline",
                           mask_origin="prompt", **bad)
        with pytest.raises(ValueError, match="temperature"):
            s.generate(_prompt(24, 2), max_tokens=16, steps=8, block_size=BS, decode_strategy="d2f_block_pipeline",
                       mask_origin="prompt", temperature=0.5)
    assert mask == cfg["mask_token_id"]
