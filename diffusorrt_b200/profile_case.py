"""Small, self-contained decode run for profiling the denoising step under a profiler.

The bench workload (Qwen3-0.6B-architecture BD3LM, long prefix) with a short generation: one
4096-token prompt and a single 32-token block (8 denoising rounds), so a profiler sees the same
kernels at the same shapes as the benchmark with few launches before them, and the device holds
about 2 GB (weights 1.19 GB, K/V cache ~0.5 GB).

    python -m diffusorrt_b200.profile_case [--prompt 4096] [--gen 32] [--rounds 8]
    python -m diffusorrt_b200.profile_case --dream [--steps 4] [--layers 28]
    python -m diffusorrt_b200.profile_case --quant --prompt 512 --gen 32

With --quant: the 4-bit affine model under bd3_fixed_quota, 16 rounds per
32-token block; every forward, prompt chunks included, runs the quantized decode linear
(gemm_decode_kernel<EPI, S, true>) in 64-row chunks: a 512-token prompt launches 8 x 28 x 4 of them
before the first denoising step.

With --dream: the Dream-7B-architecture full-canvas workload (prompt 256 + canvas 256,
entropy_count over --steps steps, each a 512-row forward); the model's synthetic weights take
~15 GB. Per step: dream_plan_kernel, embed_rows_kernel, per layer [rmsnorm, gemm_swapab (QKV),
attn_prefix, gemm_swapab (o), rmsnorm, gemm_swapab (gate/up), gemm_swapab (down)], rmsnorm,
gemm_swapab (lm_head), sel_topp_entropy_kernel, dream_commit_kernel.

Prints one JSON line: denoising steps run, kernel launches of the request and ms per step.

Kernel order, for a profiler's name filter and skip count: the prompt prefill launches one
embed_rows_kernel and two rmsnorm_bf16_kernel per layer (with the prefill linears and attention);
every denoising step then launches plan_kernel, embed_rows_kernel, per layer
[rmsnorm, gemm_decode (QKV), attn_decode, attn_merge, gemm_decode (o), rmsnorm, gemm_decode
(gate/up), gemm_decode (down)], then rmsnorm, gemm_lm_kernel (lm_head; gemm_decode for the
4-bit model), sel_pass1_kernel and commit_kernel.
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
    ap.add_argument("--dream", action="store_true", help="Dream-7B full-canvas entropy_count instead")
    ap.add_argument("--steps", type=int, default=4, help="entropy_count steps (--dream)")
    ap.add_argument("--layers", type=int, default=0, help="transformer layers (--dream; 0 = the model's 28)")
    ap.add_argument("--quant", action="store_true",
                    help="4-bit affine (group 64) linears and lm_head, bd3_fixed_quota with 16 rounds per block")
    args = ap.parse_args()
    from diffusorrt_b200 import Runtime
    from diffusorrt_b200.config import DREAM_7B, QWEN3_06B_BD3LM

    if args.dream:
        prompt_len = 256 if args.prompt == 4096 else args.prompt
        gen = 256 if args.gen == 32 else args.gen
        canvas = prompt_len + gen
        cfg = dict(DREAM_7B)
        if args.layers > 0:
            cfg["layer_count"] = args.layers
        rt = Runtime(model_config=cfg, synthetic_seed=0, device_ordinal=0, max_seq=canvas, max_prefill_rows=canvas)
        sess = rt.session({"decode_strategy": "entropy_count"})
        prompt = [int(t) for t in np.random.default_rng(0).integers(0, 151643, size=prompt_len)]
        res = sess.generate(prompt, max_tokens=gen, steps=args.steps, temperature=0.2, top_p=0.95, eps=1e-3)
        forwards = int(res["forward_count"])
        print(json.dumps({"prompt": prompt_len, "gen": gen, "forwards": forwards,
                          "kernel_launches": int(res["kernel_launches"]),
                          "decode_ms_per_step": res["decode_ms"] / max(1, forwards)}), flush=True)
        sess.close()
        rt.close()
        return

    cfg = dict(QWEN3_06B_BD3LM)
    max_seq = ((args.prompt + args.gen + 127) // 128) * 128
    engine = {"linear_quant_bits": 4, "linear_quant_group_size": 64} if args.quant else None
    rt = Runtime(model_config=cfg, synthetic_seed=0, device_ordinal=0, max_seq=max_seq,
                 max_prefill_rows=min(4096, ((args.prompt + 127) // 128) * 128), engine_config=engine)
    strategy = "bd3_fixed_quota" if args.quant else "block_threshold"
    sess = rt.session({"decode_strategy": strategy, "block_size": 32})
    prompt = [int(t) for t in np.random.default_rng(0).integers(0, 151643, size=args.prompt)]
    steps = (args.gen // 32) * (16 if args.quant else args.rounds)
    res = sess.generate(prompt, max_tokens=args.gen, steps=steps, block_size=32, decode_strategy=strategy,
                        confidence_threshold=0.9, rounds_per_block=0 if args.quant else args.rounds)
    forwards = int(res["forward_count"])
    print(json.dumps({"prompt": args.prompt, "gen": args.gen, "forwards": forwards,
                      "kernel_launches": int(res["kernel_launches"]),
                      "decode_ms_per_step": res["decode_ms"] / max(1, forwards)}), flush=True)
    sess.close()
    rt.close()


if __name__ == "__main__":
    main()
