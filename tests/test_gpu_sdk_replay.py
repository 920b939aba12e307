"""The DiffusorRT SDK's own device-session call sequences, replayed against this library on the GPU.

tests/golden/make_sdk_calls.py ran the reference SDK's ``generate_device_tokens``
(python/src/edllm/backends/device_runtime.py:108-274) with a recording session and stored every
call — start_device with the SDK's keywords (exact_kv, temperature, seed, memory budget ...),
propose_device(frontier, window_end=, frozen_prefix=) and commit_device — in sdk_calls.json. Each
call is replayed in order on a diffusorrt_b200 session opened as the SDK opens it: every call must
be accepted, and every proposal must return what the SDK's loop checks (one f64 score and one token
id per frontier row, in frontier order, and the forwarded row count: the whole window for the
cache-off BD3 shape, the uncached rows for exact K/V reuse).
"""
from __future__ import annotations

import json

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

BASE = dict(layer_count=2, hidden_size=256, attention_heads=4, num_kv_heads=2, head_dim=128, intermediate_size=512,
            vocab_size=4096, rms_norm_eps=1e-6, rope_theta=1e6, mask_token_id=4000, eos_token_id=4001)
MODELS = {
    "bd3": dict(BASE, qk_norm=True, qkv_bias=False, tied_lm_head=True, block_size=32),
    "dream": dict(BASE, qk_norm=False, qkv_bias=True, tied_lm_head=False, logits_shift=True, block_size=8,
                  mask_origin="prompt"),
}


@pytest.fixture(scope="module")
def fixture(golden_dir):
    return json.loads((golden_dir / "sdk_calls.json").read_text())


@pytest.mark.parametrize("case,model", [("bd3_fixed_quota", "bd3"), ("bd3_sampled", "bd3"),
                                        ("dream_block_threshold", "dream")])
def test_sdk_call_sequence_replays(fixture, case, model):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import Runtime

    rec = fixture["cases"][case]
    opts = rec["options"]
    vocab = fixture["vocab"]
    with Runtime(model_config=MODELS[model], max_seq=256, max_prefill_rows=128) as rt:
        rt.init_synthetic(7, linear_std=0.05, embed_std=0.5, bias_std=0.02)
        session_config = {"decode_strategy": opts["decode_strategy"], "attention_mask_kind": opts["attention_mask_kind"],
                          "block_size": opts["block_size"], "steps": opts["steps"],
                          "max_tokens": opts["max_tokens"]}
        with rt.session(session_config) as s:
            proposals = 0
            for call in rec["calls"]:
                method, args, kwargs = call["method"], call["args"], call["kwargs"]
                if method == "start_device":
                    s.start_device(*args, **kwargs)
                elif method == "propose_device":
                    frontier = args[0]
                    scores, tokens, forwarded = s.propose_device(*args, **kwargs)
                    proposals += 1
                    assert len(scores) == len(tokens) == len(frontier)
                    assert all(isinstance(v, float) and 0.0 < v <= 1.0 for v in scores)
                    assert all(isinstance(t, int) and 0 <= t < vocab for t in tokens)
                    if opts["exact_kv"]:
                        # the uncached rows, plus the Dream shift feeder row forwarded again
                        assert 1 <= forwarded <= kwargs["window_end"] + 1
                    else:
                        assert forwarded == kwargs["window_end"]  # cache-off: the whole window
                elif method == "commit_device":
                    s.commit_device(*args, **kwargs)
                else:
                    raise AssertionError(f"unexpected SDK call {method}")
            m = s.device_metrics()
    assert proposals == rec["forward_count"]
    assert m["forward_count"] == rec["forward_count"]
    assert m["committed_token_count"] == sum(len(c["args"][0]) for c in rec["calls"] if c["method"] == "commit_device")
