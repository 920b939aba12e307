"""Small, self-contained decode run for profiling the denoising step under a profiler.

The bench workload (Qwen3-0.6B-architecture BD3LM, long prefix) with a short generation: one
4096-token prompt and a single 32-token block (8 denoising rounds), so a profiler sees the same
kernels at the same shapes as the benchmark with few launches before them, and the device holds
about 2 GB (weights 1.19 GB, K/V cache ~0.5 GB).

    python -m diffusorrt_b200.profile_case [--prompt 4096] [--gen 32] [--rounds 8]

Prints one JSON line: denoising steps run, kernel launches of the request and ms per step.

Kernel order, for a profiler's name filter and skip count: the prompt prefill launches one
embed_rows_kernel and two rmsnorm_bf16_kernel per layer (with the prefill linears and attention);
every denoising step then launches plan_kernel, embed_rows_kernel, per layer
[rmsnorm, gemm_decode (QKV), attn_decode, attn_merge, gemm_decode (o), rmsnorm, gemm_decode
(gate/up), gemm_decode (down)], then rmsnorm, gemm_decode (lm_head), sel_pass1_kernel and
commit_kernel.
"""
from __future__ import annotations

import argparse
import json

import numpy as np


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--prompt", type=int, default=4096)
    ap.add_argument("--gen", type=int, default=32)
    ap.add_argument("--rounds", type=int, default=8)
    args = ap.parse_args()
    from diffusorrt_b200 import Runtime
    from diffusorrt_b200.config import QWEN3_06B_BD3LM

    cfg = dict(QWEN3_06B_BD3LM)
    max_seq = ((args.prompt + args.gen + 127) // 128) * 128
    rt = Runtime(model_config=cfg, synthetic_seed=0, device_ordinal=0, max_seq=max_seq,
                 max_prefill_rows=min(4096, ((args.prompt + 127) // 128) * 128))
    sess = rt.session({"decode_strategy": "block_threshold", "block_size": 32})
    prompt = [int(t) for t in np.random.default_rng(0).integers(0, 151643, size=args.prompt)]
    steps = (args.gen // 32) * args.rounds
    res = sess.generate(prompt, max_tokens=args.gen, steps=steps, block_size=32, decode_strategy="block_threshold",
                        confidence_threshold=0.9, rounds_per_block=args.rounds)
    forwards = int(res["forward_count"])
    print(json.dumps({"prompt": args.prompt, "gen": args.gen, "forwards": forwards,
                      "kernel_launches": int(res["kernel_launches"]),
                      "decode_ms_per_step": res["decode_ms"] / max(1, forwards)}), flush=True)
    sess.close()
    rt.close()


if __name__ == "__main__":
    main()
