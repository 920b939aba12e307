"""One rank of the tensor-parallel parity check (launched by test_gpu_tp.py through
torch.distributed.run, one process per GPU). Exits non-zero on a failed check.

Every rank holds a shard of the same seeded Dream-architecture model. Checked:
* all ranks return bit-identical window logits and final canvases (the all-reduced residual is
  replicated, so everything downstream of it is the same computation on every rank);
* the sharded window logits match the whole model on one GPU within the f32 summation-order and
  bf16 rounding tolerance, and match the CPU oracle forward as the single-GPU path does;
* entropy_count generation on the group agrees with the oracle loop on certified steps;
* the vocabulary-parallel lm_head (each rank projects its vocabulary tiles and stores them into
  every rank's logits) gives the same decode, bit for bit, as every rank projecting the whole
  vocabulary; the vocabulary (35 tiles of 128) splits unevenly over 2, 4 and 8 ranks.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

DREAM_TP = dict(layer_count=2, hidden_size=256, attention_heads=28, num_kv_heads=4, head_dim=128,
                intermediate_size=512, vocab_size=4480, qk_norm=False, qkv_bias=True, tied_lm_head=False, logits_shift=True,
                rms_norm_eps=1e-6, rope_theta=1e6, mask_token_id=4000, eos_token_id=4001, block_size=8)
STD = dict(linear_std=0.05, embed_std=0.05, bias_std=0.02)
SEED = 33
T, TOP_P, EPS = 0.2, 0.95, 1e-3


def main() -> int:
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from diffusorrt_b200 import Runtime, build
    from oracle import forward as ofwd
    from oracle import policy as opol
    from oracle import selector as osel
    from oracle.numerics import synth_weights

    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    if rank == 0:
        build.build()
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device(f"cuda:{local}"))
    dist.barrier()
    mask = DREAM_TP["mask_token_id"]
    rng = np.random.default_rng(5)
    prompt = [int(t) for t in rng.integers(0, 4000, size=48)]
    ids = prompt + [mask] * 32
    scope = [48, 49, 60, 79, 0, 20]
    gen, steps = 32, 16
    rt = Runtime(model_config=DREAM_TP, max_seq=128, max_prefill_rows=128, device_ordinal=local, tensor_parallel=True)
    rt.init_synthetic(SEED, **STD)
    with rt.session({"decode_strategy": "entropy_count"}) as s:
        win = s.execute_window(ids, scope)
        out = s.generate(prompt, max_tokens=gen, steps=steps, temperature=T, top_p=TOP_P, eps=EPS, trace_steps=steps)
    # the same request with every rank projecting the whole vocabulary: the vocabulary-parallel
    # lm_head (the default above) gathers the same logits, so trace and canvas agree bit for bit
    with rt.session({"decode_strategy": "entropy_count", "tp_vocab_parallel": False}) as s:
        out_rep = s.generate(prompt, max_tokens=gen, steps=steps, temperature=T, top_p=TOP_P, eps=EPS, trace_steps=steps)
    # the NCCL all-reduce path (sessions that do not map the peers' buffers) on the same window
    with rt.session({"decode_strategy": "entropy_count", "tp_peer_memory": False}) as s:
        win_nccl = s.execute_window(ids, scope)
    rt.close()
    logits = np.frombuffer(win.logits, dtype="<f4").reshape(win.n_rows, win.n_vocab)
    logits_nccl = np.frombuffer(win_nccl.logits, dtype="<f4").reshape(win.n_rows, win.n_vocab)
    allx = [None] * world
    dist.all_gather_object(allx, (logits.tobytes(), out["x"], out["trace"]))
    ok = True
    if out_rep["x"] != out["x"] or out_rep["trace"] != out["trace"]:
        print(f"rank {rank}: vocabulary-parallel and replicated lm_head decodes differ", flush=True)
        ok = False
    nerr = float(np.abs(logits - logits_nccl).max())
    if nerr > 5e-3 * float(np.abs(logits).max()):
        print(f"rank {rank}: peer-memory and NCCL reductions differ by {nerr:.3e}", flush=True)
        ok = False
    if rank == 0:
        print(f"max |peer - nccl| = {nerr:.3e}", flush=True)
        for r in range(1, world):
            if allx[r][0] != allx[0][0] or allx[r][1] != allx[0][1]:
                print(f"rank {r} differs from rank 0", flush=True)
                ok = False
        whole = Runtime(model_config=DREAM_TP, max_seq=128, max_prefill_rows=128, device_ordinal=local)
        whole.init_synthetic(SEED, **STD)
        with whole.session({"decode_strategy": "entropy_count"}) as s:
            ref = np.frombuffer(s.execute_window(ids, scope).logits, dtype="<f4").reshape(len(scope), -1)
        whole.close()
        scale = float(np.abs(ref).max())
        err = float(np.abs(logits - ref).max())
        print(f"world {world}: max |tp - whole| = {err:.3e} (scale {scale:.3f})", flush=True)
        if err > 5e-3 * scale:
            ok = False
        w = synth_weights(DREAM_TP, SEED, **STD)
        want = ofwd.forward_mlx(w, DREAM_TP, ids, bidirectional=True, output_rows=ofwd.dream_raw_rows(scope))
        oerr = float(np.abs(logits - want).max())
        print(f"max |tp - oracle| = {oerr:.3e}", flush=True)
        if oerr > 0.02 * float(np.abs(want).max()):
            ok = False
        c = opol.Canvas(list(prompt) + [mask] * gen, len(prompt), mask, DREAM_TP["eos_token_id"])
        pol = opol.EntropyCount(eps=EPS, steps=steps)
        certified = 0
        for tr in out["trace"]:
            plan = pol.plan(c, tr["step"])
            if plan.frontier != tr["frontier"]:
                print("frontier mismatch", tr["step"], flush=True)
                ok = False
                break
            lg = osel.exclude_mask_token(ofwd.forward_mlx(w, DREAM_TP, c.x, bidirectional=True,
                                                          output_rows=ofwd.dream_raw_rows(plan.frontier)), mask)
            conf, tok = osel.neg_entropy_rows(lg, temperature=T, top_p=TOP_P)
            rows = pol.select(conf)
            order = np.sort(np.asarray(conf, np.float64))[::-1]
            k = len(rows)
            gap = abs(order[k - 1] - order[k]) / max(abs(order[k - 1]), 1e-30) if k < len(order) else 1.0
            if tr["tie"] == 0 and gap > 0.05:
                if sorted(rows) != tr["chosen"]:
                    print(f"step {tr['step']}: chosen rows differ on a clear margin ({gap:.3g})", flush=True)
                    ok = False
                certified += 1
            for i in tr["chosen"]:
                c.x[plan.frontier[i]] = tr["tokens"][i]
        print(f"certified steps: {certified} of {len(out['trace'])}", flush=True)
        if c.x != out["x"] or certified < max(2, len(out["trace"]) // 5):
            ok = False
    flag = torch.tensor([0 if ok else 1], device=f"cuda:{local}")
    dist.all_reduce(flag, op=dist.ReduceOp.MAX)
    dist.destroy_process_group()
    return int(flag.item())


if __name__ == "__main__":
    sys.exit(main())
