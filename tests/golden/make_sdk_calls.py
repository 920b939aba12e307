"""Record the device-session calls the DiffusorRT SDK makes, for replay against this library.

Runs the reference SDK's own ``generate_device_tokens`` (python/src/edllm/backends/device_runtime.py)
with a recording session that answers every proposal from a deterministic stand-in (no model), and
writes each call the SDK made — method, positional arguments and keywords, in order — plus what the
stand-in returned, to sdk_calls.json next to this script. tests/test_gpu_sdk_replay.py replays the
calls against diffusorrt_b200.Runtime sessions on the GPU. The reference tree is only read; nothing
here runs on the GPU box.

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_sdk_calls.py --reference /path/to/reference
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

VOCAB, MASK, EOS = 4096, 4000, 4001


class RecordingSession:
    """Stand-in device session: proposals score each frontier row from a hash of (forward, position)
    and propose a non-MASK token; every call is logged."""

    def __init__(self):
        self.calls = []
        self.forwards = 0

    def _log(self, name, args, kwargs, result=None):
        self.calls.append({"method": name, "args": [list(a) if isinstance(a, (list, tuple)) else a for a in args],
                           "kwargs": {k: (list(v) if isinstance(v, (list, tuple)) else v) for k, v in kwargs.items()},
                           "result": result})

    def start_device(self, x, **kwargs):
        self._log("start_device", [list(x)], kwargs)

    def propose_device(self, frontier, **kwargs):
        rng = np.random.default_rng(1000 + self.forwards)
        self.forwards += 1
        scores = [float(v) for v in rng.uniform(0.05, 0.99, size=len(frontier))]
        tokens = [int(v) for v in rng.integers(0, MASK, size=len(frontier))]
        forwarded = int(kwargs["window_end"])
        self._log("propose_device", [list(frontier)], kwargs, [scores, tokens, forwarded])
        return scores, tokens, forwarded

    def commit_device(self, positions, token_ids):
        self._log("commit_device", [list(positions), list(token_ids)], {})


CASES = {
    # BD3LM (d2f_hybrid graph, absolute blocks, no K/V reuse), the cuda_native defaults for it
    "bd3_fixed_quota": dict(prompt_len=64, max_tokens=64, steps=64, block_size=32, decode_strategy="bd3_fixed_quota",
                            attention_mask_kind="d2f_hybrid", exact_kv=False, requires_prompt_block_alignment=True),
    "bd3_sampled": dict(prompt_len=32, max_tokens=64, steps=32, block_size=32, decode_strategy="bd3_fixed_quota",
                        attention_mask_kind="d2f_hybrid", exact_kv=False, requires_prompt_block_alignment=True,
                        temperature=0.7, seed=5),
    # Dream D2F (exact K/V reuse, prompt-relative blocks of 8), the shipped CUDA profile's policy
    "dream_block_threshold": dict(prompt_len=24, max_tokens=24, steps=24, block_size=8,
                                  decode_strategy="block_threshold", attention_mask_kind="d2f_hybrid", exact_kv=True,
                                  confidence_threshold=0.9),
}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DIFFUSORRT_REFERENCE"),
                    help="checkout of the reference project (or set DIFFUSORRT_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference checkout with --reference or DIFFUSORRT_REFERENCE")
    sys.path.insert(0, str(Path(args.reference) / "python" / "src"))
    sys.dont_write_bytecode = True
    from edllm.backends.device_runtime import generate_device_tokens

    out = {"vocab": VOCAB, "mask_token_id": MASK, "eos_token_id": EOS, "cases": {}}
    for name, case in CASES.items():
        case = dict(case)
        prompt = [int(t) for t in np.random.default_rng(len(name)).integers(0, MASK, size=case.pop("prompt_len"))]
        session = RecordingSession()
        result = generate_device_tokens(session, prompt, mask_token_id=MASK, eos_token_id=EOS, **case)
        out["cases"][name] = {"options": case, "prompt": prompt, "calls": session.calls,
                              "forward_count": int(result.forward_count)}
    (HERE / "sdk_calls.json").write_text(json.dumps(out, indent=1))
    print("sdk call fixture written to", HERE / "sdk_calls.json")


if __name__ == "__main__":
    main()
