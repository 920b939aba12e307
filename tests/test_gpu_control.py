"""Control paths of the device session on the GPU, through the C ABI:

* failure handling: a bounded device wait that nothing satisfies (the wait a tensor-parallel
  reducer makes for a stopped peer) returns DRT_DEVICE_TIMEOUT, and the same session then serves a
  normal propose with unchanged results — no GPU fault is raised;
* EOS: BD3's stop at a block boundary once EOS is in the canvas
  (BD3FixedQuotaCommit.plan, python/src/edllm/backends/diffusion_runtime.py:1305-1309) and the
  finalize fields (MaskState.finalize, :526-558), on the device loop against the host loop with
  the oracle policy;
* exact_kv: reuse of the frozen prefix's K/V (exact_kv=True) and its recomputation
  (exact_kv=False) give the same scores up to the bf16 rounding of K/V made by different kernels,
  and the forwarded row counts of the two shapes; the
  bidirectional session refuses exact K/V as the reference does (device_runtime.py:125-126).
"""
from __future__ import annotations

import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import policy as opol  # noqa: E402

pytestmark = pytest.mark.gpu

SMALL = dict(layer_count=2, hidden_size=256, attention_heads=4, num_kv_heads=2, head_dim=128,
             intermediate_size=512, vocab_size=4096, qk_norm=True, qkv_bias=False, tied_lm_head=True,
             rms_norm_eps=1e-6, rope_theta=1e6, mask_token_id=4000, eos_token_id=4001, block_size=32)
STD = dict(linear_std=0.05, embed_std=0.5)


@pytest.fixture(scope="module")
def rt():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import Runtime, build

    build.build()
    r = Runtime(model_config=SMALL, max_seq=512, max_prefill_rows=256)
    r.init_synthetic(3, **STD)
    yield r
    r.close()


@pytest.fixture(scope="module")
def rt_untied():
    """An untied lm_head, so the masked rows commit varied tokens (a tied head at this embedding
    scale predicts MASK at every masked row)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import Runtime, build

    build.build()
    r = Runtime(model_config=dict(SMALL, tied_lm_head=False), max_seq=512, max_prefill_rows=256)
    r.init_synthetic(3, **STD)
    yield r
    r.close()


def _prompt(n, seed, vocab=4000):
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, size=n)]


def test_expired_peer_wait_reports_timeout_and_session_survives(rt):
    from diffusorrt_b200.runtime import DeviceTimeout

    mask = SMALL["mask_token_id"]
    x = _prompt(64, 5) + [mask] * 32
    frontier = list(range(64, 96))
    with rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
        s.start_device(x, prompt_len=0, block_size=32, mask_token_id=mask, exact_kv=True, steps=32)
        before = s.propose_device(frontier, window_end=96, frozen_prefix=64)
        t0 = time.monotonic()
        with pytest.raises(DeviceTimeout):
            s.peer_wait_drill()
        waited = time.monotonic() - t0
        assert 1.5 <= waited <= 30.0, waited  # the 2 s device limit, then a clean return
        after = s.propose_device(frontier, window_end=96, frozen_prefix=64)
        assert after[0] == before[0] and after[1] == before[1]
        # a second drill behaves the same (the status word was cleared)
        with pytest.raises(DeviceTimeout):
            s.peer_wait_drill()
        s.commit_device([64], [after[1][0]])


def _host_loop_eos(s, prompt, gen, steps, eos):
    mask = SMALL["mask_token_id"]
    x = list(prompt) + [mask] * gen
    s.start_device(x, prompt_len=0, block_size=32, mask_token_id=mask, exact_kv=True, steps=steps)
    c = opol.Canvas(list(x), len(prompt), mask, eos)
    pol = opol.BD3FixedQuota(block_size=32, steps=steps, prompt_len=len(prompt), gen_len=gen)
    forwards = 0
    for step in range(pol.iteration_limit):
        plan = pol.plan(c, step)
        if plan.action == "stop":
            break
        if plan.action == "skip":
            continue
        frozen = (min(plan.frontier) // 32) * 32
        sc, tok, _ = s.propose_device(plan.frontier, window_end=plan.window_end, frozen_prefix=frozen)
        forwards += 1
        rows = pol.select(np.asarray(sc))
        pos = [plan.frontier[r] for r in rows]
        s.commit_device(pos, [tok[r] for r in rows])
        for p, r in zip(pos, rows):
            c.x[p] = tok[r]
    return c, forwards


def test_eos_stops_at_block_boundary_and_finalizes(rt_untied):
    rt = rt_untied
    prompt = _prompt(64, 17)
    gen, steps = 96, 48  # 3 blocks, 16 rounds each, quota 2
    with rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
        free = s.generate(prompt, max_tokens=gen, steps=steps, block_size=32, trace_steps=64)
    # EOS := the first non-MASK token the device commits in the first generated block before its last
    # round, so EOS lands mid-block while other rows of the block are still masked
    spb = 16
    eos = None
    for tr in free["trace"][: spb - 1]:
        picks = [tr["tokens"][r] for r in tr["chosen"] if tr["tokens"][r] != SMALL["mask_token_id"]]
        if picks:
            eos = picks[0]
            break
    assert eos is not None
    with rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
        dev = s.generate(prompt, max_tokens=gen, steps=steps, block_size=32, eos_token_id=eos, trace_steps=64)
    with rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
        canvas, forwards = _host_loop_eos(s, prompt, gen, steps, eos)
    # the block in which EOS first appears is finished, the decode stops at the next boundary
    assert dev["stopped"] == 1
    assert dev["forward_count"] == forwards == spb
    assert dev["x"] == canvas.x
    assert dev["x"][96:] == [SMALL["mask_token_id"]] * 64  # later blocks never forwarded
    assert dev["x"][64:96] == free["x"][64:96]  # the finished block is the EOS-free decode's
    want = canvas.finalize()
    for key in ("visible_token_ids", "hit_eos", "remaining_mask_count", "finish_reason"):
        assert dev[key] == want[key], key
    assert dev["hit_eos"] is True
    assert dev["finish_reason"] == want["finish_reason"]


def test_exact_kv_reuse_equals_recompute(rt):
    mask = SMALL["mask_token_id"]
    prompt = _prompt(96, 23)
    x = prompt + [mask] * 64
    runs = {}
    for exact in (True, False):
        with rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
            s.start_device(x, prompt_len=0, block_size=32, mask_token_id=mask, exact_kv=exact, steps=64)
            out = []
            for lo in (96, 128):
                frontier = list(range(lo, lo + 32))
                sc, tok, fwd = s.propose_device(frontier, window_end=lo + 32, frozen_prefix=lo)
                s.commit_device(frontier, tok)
                out.append((sc, tok, fwd))
            runs[exact] = out
    # the first forward is the same computation in both modes
    assert runs[True][0][1] == runs[False][0][1]
    np.testing.assert_array_equal(np.asarray(runs[True][0][0]), np.asarray(runs[False][0][0]))
    # the second reuses the prefix K/V or recomputes it through the prefill kernels: the same values
    # up to the bf16 rounding of K/V computed by different kernels
    (sc1, tok1, _), (sc0, tok0, _) = runs[True][1], runs[False][1]
    assert np.mean(np.asarray(tok1) == np.asarray(tok0)) >= 0.9
    np.testing.assert_allclose(np.asarray(sc1), np.asarray(sc0), rtol=0.05)
    # reuse forwards the uncached rows (the finished block's K/V is recomputed with its final tokens
    # at the next forward, the exact-D2F pattern); recomputation forwards the whole window each time
    assert [r[2] for r in runs[True]] == [128, 64]
    assert [r[2] for r in runs[False]] == [128, 160]


def test_bidirectional_session_refuses_exact_kv():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import Runtime

    cfg = dict(SMALL, qk_norm=False, qkv_bias=True, tied_lm_head=False)
    with Runtime(model_config=cfg, max_seq=128, max_prefill_rows=128) as r:
        r.init_synthetic(1, linear_std=0.05, embed_std=0.05, bias_std=0.02)
        with r.session({"decode_strategy": "entropy_count"}) as s:
            x = _prompt(24, 3) + [SMALL["mask_token_id"]] * 8
            with pytest.raises(ValueError):
                s.start_device(x, prompt_len=24, block_size=8, mask_token_id=SMALL["mask_token_id"], exact_kv=True,
                               steps=8)
            with pytest.raises(NotImplementedError):
                s.start_device(x, prompt_len=24, block_size=8, mask_token_id=SMALL["mask_token_id"], exact_kv=False,
                               steps=8)
