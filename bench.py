#!/usr/bin/env python
"""Benchmark of the denoising-decode hot path (one JSON line on rank 0).

Workload (default): the long-prefix BD3LM configuration — Qwen3-0.6B architecture with seeded
random bf16 weights, 4096-token random prompt, 512 generated tokens, block 32, confidence-
threshold unmask (p >= 0.9, at least one per step) with a budget of 8 denoising rounds per
block (16 blocks x 8 = 128 denoising steps), batch 1 per GPU; with N GPUs, N independent
seeded requests run one per GPU (request-parallel, weak scaling, no collective on the data path).

One bench step = one complete request: prompt upload, prefill, every denoising step (forward,
selector, policy, commit on the GPU), canvas download.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload cfg1|cfg0|cfg2|cfg3|cfg4|d2f|d2f_bt]

--workload cfg0 / cfg3: BASELINE configs[0] / [3] (cfg3: the cfg0 model with 4-bit affine, group 64
linears and lm_head, prompt 512, 256 new tokens, 2 commits per round).

--workload cfg2 is BASELINE configs[2]: Dream-7B architecture (28 layers, hidden 3584, 28/4 heads,
intermediate 18944, vocab 152064, q/k/v bias, untied lm_head), 256-token prompt plus a 256-token
all-MASK canvas, entropy_count over 256 steps (NegEntropy T 0.2, top_p 0.95, eps 1e-3, MASK
excluded): every step forwards the whole 512-row canvas with bidirectional attention. With N > 1
GPUs the one request runs tensor-parallel over the group (heads and MLP sharded, the row-split
linears reduced over NVLink peer memory, the lm_head split by vocabulary), strong scaling; its
roofline is tensor-core FLOP/s.

--workload d2f (not a BASELINE config): the reference's exact active-window preset on the Dream-7B
architecture: D2F graph with the prompt as the mask origin, d2f_block_pipeline (block 8, tau_conf
0.8, tau_add 0.1, tau_act 0.95), 256-token prompt, 256 new tokens; HBM roofline of the step.
--workload d2f_bt: the same model and canvas under the reference's shipped Dream CUDA profile,
block_threshold (tau 0.9) over blocks of 8 with exact K/V.

--workload cfg4 is the isolated unmask-selector microbenchmark: fp32 logits
[B, L, 151936] ~ N(0, 3^2) from a seed, a Bernoulli(0.5) mask of masked positions, max-prob and
entropy confidence over the masked rows, then top-k (k = 1, 4, 8) and threshold-0.9 choices per
batch item; reported as HBM GB/s of the logits the selector must read (the masked rows once).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "generated tokens/sec/request and ms per denoising step at 1/2/4/8 B200"

WORKLOADS = {
    # long prefix, block threshold with a per-block round budget.
    "cfg1": dict(prompt=4096, gen=512, block=32, strategy="block_threshold", steps=128, rounds=8, tau=0.9),
    # prompt 64, 128 new tokens, 32 rounds per block, top-1 fixed quota.
    "cfg0": dict(prompt=64, gen=128, block=32, strategy="bd3_fixed_quota", steps=128, rounds=0, tau=0.9),
    # the cfg0 model with 4-bit affine (group 64) layer linears and lm_head,
    # prompt 512, 256 new tokens, 128 steps = 8 blocks x 16 rounds, 2 commits per round.
    "cfg3": dict(prompt=512, gen=256, block=32, strategy="bd3_fixed_quota", steps=128, rounds=0, tau=0.9, quant=True),
    # Not a BASELINE config: the reference's exact active-window preset (d2f_block_pipeline, block 8,
    # tau_conf 0.8, tau_add 0.1, tau_act 0.95, exact prefix K/V) on the Dream-7B architecture, prompt
    # 256, 256 new tokens (the D2F block-pipeline row's measurement).
    "d2f": dict(model="dream", prompt=256, gen=256, block=8, strategy="d2f_block_pipeline", steps=256, rounds=0,
                tau=0.8, tau_add=0.1, tau_act=0.95, origin="prompt"),
    # Not a BASELINE config: the reference's shipped Dream CUDA profile (cuda_profile.py:63-82, 96-119):
    # block_threshold (tau 0.9, at least one per step) over blocks of 8 on the D2F graph, exact K/V.
    "d2f_bt": dict(model="dream", prompt=256, gen=256, block=8, strategy="block_threshold", steps=256, rounds=0,
                   tau=0.9, origin="prompt"),
}


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() in ("active", "1"):
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def _weight_bytes(cfg: dict, quant: bool = False) -> int:
    """Weight bytes one denoising step streams: bf16 linears and lm_head, or (quant) their 4-bit
    nibbles plus a bf16 scale and bias per group of 64 inputs."""
    H, I, V = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    qd, kd = cfg["attention_heads"] * cfg["head_dim"], cfg["num_kv_heads"] * cfg["head_dim"]
    per_layer = H * (qd + 2 * kd) + qd * H + 2 * I * H + I * H
    params = cfg["layer_count"] * per_layer + V * H
    if quant:
        return params // 2 + (params // 64) * 4
    return 2 * params


def _kv_bytes_per_pos(cfg: dict) -> int:
    return cfg["layer_count"] * 2 * cfg["num_kv_heads"] * cfg["head_dim"] * 2


def _algorithmic_bytes(cfg: dict, w: dict, trace_kv: list[int]) -> float:
    """Average HBM bytes one denoising step must move: every weight once, the visible K/V of
    the forwarded rows once, the active block's K/V written once."""
    wb = _weight_bytes(cfg, bool(w.get("quant")))
    kvp = _kv_bytes_per_pos(cfg)
    if not trace_kv:
        return float(wb)
    kv = float(np.mean(trace_kv)) * kvp
    return wb + kv + w["block"] * kvp


def _measured_traffic(alg_bytes: float) -> float | None:
    """DRAM bytes per denoising step from the committed ncu capture (profiles/), scaled from the
    captured K/V length to this run's algorithmic bytes (traffic grows with the bytes streamed)."""
    p = ROOT / "profiles" / "decode_step_cfg1_traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    return float(d["dram_bytes_per_step"]) * alg_bytes / float(d["algorithmic_bytes_per_step"])


def _frontier_stats(sess, prompt, w, probe) -> dict:
    """Logit scale and decision margins at the frontier (outside the timed region): the std of the
    first block's frontier logits (one window forward), the spread of the rows' max-prob confidences,
    and per step the gap between the best and second-best frontier confidence (the margin of the
    block-threshold / top-k choice) over the traced request."""
    mask = int(sess.runtime.config["mask_token_id"])
    n = len(prompt)
    scope = list(range(n, n + w["block"]))
    origin = n if w.get("origin") == "prompt" else 0
    res = sess.execute_window(list(prompt) + [mask] * w["block"], scope, mask_geometry=(origin, w["block"]))
    logits = np.frombuffer(res.logits, dtype="<f4").reshape(res.n_rows, res.n_vocab).astype(np.float64)
    x = logits - logits.max(axis=1, keepdims=True)
    max_prob = 1.0 / np.exp(x).sum(axis=1)
    gaps = []
    for t in probe["trace"]:
        sc = sorted(t["scores"], reverse=True)
        if len(sc) >= 2:
            gaps.append(sc[0] - sc[1])
    q = lambda a, v: float(np.quantile(a, v)) if len(a) else None  # noqa: E731
    return {"frontier_logit_std": round(float(logits.std()), 5),
            "frontier_max_prob": {"p10": q(max_prob, 0.1), "p50": q(max_prob, 0.5), "p90": q(max_prob, 0.9)},
            "step_conf_gap_top2": {"p10": q(gaps, 0.1), "p50": q(gaps, 0.5), "p90": q(gaps, 0.9), "steps": len(gaps)}}


def _run_ours(args, world, rank, local) -> dict | None:
    import torch

    from diffusorrt_b200 import Runtime, build
    from diffusorrt_b200.config import DREAM_7B, QWEN3_06B_BD3LM

    if rank == 0:
        build.build()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        build.build()
    torch.cuda.set_device(local)
    w = WORKLOADS[args.workload]
    cfg = dict(DREAM_7B if w.get("model") == "dream" else QWEN3_06B_BD3LM)
    max_seq = ((w["prompt"] + w["gen"] + 127) // 128) * 128
    engine = {"linear_quant_bits": 4, "linear_quant_group_size": 64} if w.get("quant") else None
    rt = Runtime(model_config=cfg, synthetic_seed=0, device_ordinal=local, max_seq=max_seq,
                 max_prefill_rows=min(4096, ((w["prompt"] + 127) // 128) * 128), engine_config=engine)
    sess = rt.session({"decode_strategy": w["strategy"], "block_size": w["block"]})
    prompt = [int(t) for t in np.random.default_rng(rank).integers(0, 151643, size=w["prompt"])]

    extra = {}
    if w["strategy"] == "d2f_block_pipeline":
        extra = dict(add_threshold=w["tau_add"], activate_threshold=w["tau_act"])
    if "origin" in w:
        extra["mask_origin"] = w["origin"]

    def request(trace=0):
        return sess.generate(prompt, max_tokens=w["gen"], steps=w["steps"], block_size=w["block"],
                             decode_strategy=w["strategy"], confidence_threshold=w["tau"],
                             rounds_per_block=w["rounds"], trace_steps=trace, **extra)

    for _ in range(args.warmup):
        request()
    probe = request(trace=256)  # one traced request: per-step K/V lengths for the roofline
    kv_lens = [max(t["frontier"]) // w["block"] * w["block"] + w["block"] for t in probe["trace"]]
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    results = []
    with ClockSampler(local) as clocks:
        wall0 = time.perf_counter()
        for _ in range(args.steps):
            results.append(request())
        torch.cuda.synchronize()
        wall = time.perf_counter() - wall0
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    dev_ms = float(np.mean([r["prefill_ms"] + r["decode_ms"] for r in results]))
    e2e_ms = float(np.mean([r["total_ms"] for r in results]))
    dec_ms = float(np.mean([r["decode_ms"] / max(1, r["forward_count"]) for r in results]))
    pre_ms = float(np.mean([r["prefill_ms"] for r in results]))
    host_ms = float(np.mean([r["host_enqueue_ms"] for r in results]))
    committed = float(np.mean([r["committed_token_count"] for r in results]))
    forwards = float(np.mean([r["forward_count"] for r in results]))
    stats = torch.tensor([dev_ms, e2e_ms, dec_ms, pre_ms], dtype=torch.float64, device=f"cuda:{local}")
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    dev_ms, e2e_ms, dec_ms, pre_ms = (float(v) for v in stats.tolist())
    margins = _frontier_stats(sess, prompt, w, probe) if rank == 0 else None
    sess.close()
    rt.close()
    if rank != 0:
        return None
    peaks = _peaks()
    alg = _algorithmic_bytes(cfg, w, kv_lens)
    achieved = alg / (dec_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC,
        "value": round(world * committed / (dev_ms * 1e-3), 3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dev_ms, 4),
        "ms_per_denoising_step": round(dec_ms, 5),
        "tokens_per_s_per_request": round(committed / (dev_ms * 1e-3), 3),
        "prefill_ms": round(pre_ms, 4),
        "host_enqueue_ms_per_request": round(host_ms, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded random-init weights and prompts)",
        "config": {"workload": f"{args.workload}: {'Dream-7B-arch D2F' if w.get('model') == 'dream' else 'Qwen3-0.6B-arch BD3LM'}"
                               f"{' (4-bit affine g64 linears + lm_head)' if w.get('quant') else ''}, "
                               f"prompt {w['prompt']}, gen {w['gen']}, block {w['block']}, {w['strategy']}"
                               + (f" tau {w['tau']} rounds/block {w['rounds']}" if w["strategy"] == "block_threshold" else
                                  f" tau_conf {w['tau']} tau_add {w['tau_add']} tau_act {w['tau_act']} steps {w['steps']}"
                                  if w["strategy"] == "d2f_block_pipeline" else f" steps {w['steps']}"),
                   "requests_per_gpu": 1, "parallelism": f"request-parallel x{world}",
                   "committed_tokens_per_request": committed, "denoising_steps_per_request": forwards,
                   "l2": (f"inputs larger than L2: {_weight_bytes(cfg, bool(w.get('quant'))) / 1e9:.2f} GB of weights "
                          "streamed every denoising step"),
                   "frontier": margins},
        "roofline": {"bound": "hbm", "kernel": "one denoising step (CUDA graph of the step's kernels)",
                     "weights": "4-bit affine" if w.get("quant") else "bf16",
                     "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                     "algorithmic_bytes_per_step": int(alg),
                     "traffic": (int(_measured_traffic(alg)) if _measured_traffic(alg) and not w.get("quant")
                                 and w.get("model") != "dream" else None),
                     "traffic_note": ("DRAM bytes per step from profiles/decode_step_cfg1_traffic.json scaled to this K/V length"
                                      if w.get("model") != "dream" and not w.get("quant") else None)},
        "e2e": {"value": round(world * committed / (e2e_ms * 1e-3), 3), "unit": "tokens/s",
                "h2d_bytes_per_step": 4 * (w["prompt"] + w["gen"]),
                "d2h_bytes_per_step": 4 * (w["prompt"] + w["gen"]) + 512},
        "gpu_launches": int(results[-1]["kernel_launches"]) * args.steps,
        "clocks": clocks.summary(),
        "wall_s": round(wall, 3),
    }
    return line


DREAM = dict(prompt=256, gen=256, steps=256, temperature=0.2, top_p=0.95, eps=1e-3)


def _dream_flops(cfg: dict, canvas: int, n_frontier: float) -> float:
    """Algorithmic FLOPs of one full-canvas step: every layer linear over the canvas, QK^T and PV
    over the canvas (bidirectional), lm_head over the frontier rows."""
    H, I, V, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"], cfg["layer_count"]
    qd, kd = cfg["attention_heads"] * cfg["head_dim"], cfg["num_kv_heads"] * cfg["head_dim"]
    per_layer = H * (qd + 2 * kd) + qd * H + 3 * I * H
    lin = 2.0 * canvas * per_layer * L
    attn = 2.0 * 2.0 * canvas * canvas * qd * L
    head = 2.0 * n_frontier * V * H
    return lin + attn + head


def _run_dream(args, world, rank, local) -> dict | None:
    """cfg2: Dream-7B-architecture full-canvas entropy_count decode, one request per GPU."""
    import torch

    from diffusorrt_b200 import Runtime, _lib, build
    from diffusorrt_b200.config import DREAM_7B

    if rank == 0:
        build.build()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        build.build()
    torch.cuda.set_device(local)
    cfg = dict(DREAM_7B)
    d = DREAM
    canvas = d["prompt"] + d["gen"]
    # one request, tensor-parallel over the group (heads and MLP sharded, NCCL all-reduce)
    tp = world > 1
    rt = Runtime(model_config=cfg, synthetic_seed=0, device_ordinal=local, max_seq=canvas, max_prefill_rows=canvas,
                 tensor_parallel=tp)
    sess = rt.session({"decode_strategy": "entropy_count"})
    prompt = [int(t) for t in np.random.default_rng(0).integers(0, 151643, size=d["prompt"])]

    def request():
        return sess.generate(prompt, max_tokens=d["gen"], steps=d["steps"], temperature=d["temperature"],
                             top_p=d["top_p"], eps=d["eps"])

    for _ in range(args.warmup):
        request()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    results = []
    with ClockSampler(local) as clocks:
        wall0 = time.perf_counter()
        for _ in range(args.steps):
            results.append(request())
        torch.cuda.synchronize()
        wall = time.perf_counter() - wall0
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    dev_ms = float(np.mean([r["decode_ms"] for r in results]))
    e2e_ms = float(np.mean([r["total_ms"] for r in results]))
    forwards = float(np.mean([r["forward_count"] for r in results]))
    committed = float(np.mean([r["committed_token_count"] for r in results]))
    stats = torch.tensor([dev_ms, e2e_ms], dtype=torch.float64, device=f"cuda:{local}")
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    dev_ms, e2e_ms = (float(v) for v in stats.tolist())
    sess.close()
    rt.close()
    if rank != 0:
        return None
    # frontier sizes of the proceeding steps, from the host schedule the device follows
    import ctypes
    sched = (ctypes.c_int32 * d["steps"])()
    _lib.check(_lib.load().drt_entropy_count_schedule(d["gen"], d["steps"], d["eps"], sched))
    left, fronts = d["gen"], []
    for k in sched:
        if k > 0:
            fronts.append(left)
            left -= k
    flops = _dream_flops(cfg, canvas, float(np.mean(fronts)))
    ms_step = dev_ms / max(1.0, forwards)
    achieved = flops / (ms_step * 1e-3) / 1e12
    pk = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(pk.get("bf16_tflops_sustained", 1400.0))
    return {
        "metric": METRIC,
        "value": round(committed / (dev_ms * 1e-3), 3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dev_ms, 3),
        "ms_per_denoising_step": round(ms_step, 4),
        "tokens_per_s_per_request": round(committed / (dev_ms * 1e-3), 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded random-init weights and prompts)",
        "config": {"workload": (f"cfg2: Dream-7B-arch full-canvas masked diffusion, prompt {d['prompt']} + canvas "
                                f"{d['gen']}, {d['steps']} steps, entropy_count (NegEntropy T {d['temperature']}, "
                                f"top_p {d['top_p']}, eps {d['eps']}), MASK excluded, argmax tokens"),
                   "requests": 1, "parallelism": f"tp{world}" if tp else "single GPU",
                   "committed_tokens_per_request": committed, "denoising_steps_per_request": forwards,
                   "l2": "inputs larger than L2: 15.2 GB of weights (per group) streamed every denoising step"},
        "roofline": {"bound": "tensor", "kernel": "one full-canvas denoising step (CUDA graph of the step's kernels)",
                     "achieved": round(achieved, 1), "peak": round(peak * world, 1), "unit": "TFLOP/s",
                     "frac": round(achieved / (peak * world), 4),
                     "peak_source": "measured (sustained)" if pk else "fallback",
                     "algorithmic_flops_per_step": int(flops), "traffic": None},
        "e2e": {"value": round(committed / (e2e_ms * 1e-3), 3), "unit": "tokens/s",
                "h2d_bytes_per_step": 4 * canvas, "d2h_bytes_per_step": 4 * canvas + 64},
        "gpu_launches": int(results[-1]["kernel_launches"]) * args.steps,
        "clocks": clocks.summary(),
        "wall_s": round(wall, 3),
    }


def _cpu_dream_baseline(sample_rows: int = 4) -> dict:
    """The reference's CPU algorithm for one cfg2 step, timed in pieces on this host: the float64
    spec forward of one Dream-7B layer over the 512-row canvas (scaled to 28 layers), the float64
    lm_head over a vocabulary slice (scaled to the full vocabulary and the mean frontier), and the
    top-p NegEntropy selector on a few rows (scaled to the frontier)."""
    from oracle import forward as ofwd
    from oracle import selector as osel
    from oracle.numerics import synth_weights

    from diffusorrt_b200.config import DREAM_7B

    cfg = dict(DREAM_7B)
    canvas, front = DREAM["prompt"] + DREAM["gen"], DREAM["gen"] / 2.0
    small_v = 2048
    sub = dict(cfg, layer_count=1, vocab_size=small_v)
    wts = synth_weights(sub, 0, linear_std=0.02, embed_std=0.02, bias_std=0.02)
    cache = {k: np.asarray(v, dtype=np.float64) for k, v in wts.items()}
    ids = [int(t) for t in np.random.default_rng(0).integers(0, small_v, size=canvas)]
    t0 = time.perf_counter()
    ofwd.forward_fp64(wts, sub, ids, bidirectional=True, output_rows=[0], cast=lambda k: cache.get(k))
    t_layer = time.perf_counter() - t0
    H, V = cfg["hidden_size"], cfg["vocab_size"]
    rng = np.random.default_rng(1)
    w_slice = rng.standard_normal((V // 16, H))
    x = rng.standard_normal((16, H))
    t1 = time.perf_counter()
    _ = x @ w_slice.T
    t_head = (time.perf_counter() - t1) * 16 * (front / 16)
    logits = (rng.standard_normal((sample_rows, V)) * 3).astype(np.float32)
    t2 = time.perf_counter()
    osel.neg_entropy_rows(logits, temperature=DREAM["temperature"], top_p=DREAM["top_p"])
    t_sel = (time.perf_counter() - t2) * front / sample_rows
    step_s = t_layer * cfg["layer_count"] + t_head + t_sel
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    return {"step_s": step_s, "ms_per_denoising_step": step_s * 1e3, "cores": cores,
            "sample": (f"one cfg2 step: 1 of 28 Dream-7B layers (float64 spec forward, {canvas} rows, bidirectional) "
                       f"scaled to 28; lm_head on 16 rows x V/16 scaled to {front:.0f} rows x V; top-p NegEntropy on "
                       f"{sample_rows} rows scaled to {front:.0f}; measured {t_layer + (t_head + t_sel) / 16:.1f} s")}


def _cpu_baseline(args, sample_layers: int = 1) -> dict:
    """The reference's CPU algorithm (float64 executable-spec forward over the whole window,
    float64 max-prob selector) for one denoising step of the workload, timed on this host."""
    from oracle import forward as ofwd
    from oracle import selector as osel
    from oracle.numerics import synth_tensor, layer_tensor_id, TID_EMBED

    from diffusorrt_b200.config import QWEN3_06B_BD3LM

    w = WORKLOADS[args.workload]
    cfg = dict(QWEN3_06B_BD3LM)
    L = cfg["layer_count"]
    H, nq, nkv, hd, I, V = (cfg[k] for k in ("hidden_size", "attention_heads", "num_kv_heads", "head_dim",
                                             "intermediate_size", "vocab_size"))
    sub = dict(cfg, layer_count=sample_layers)
    wts = {"model.embed_tokens.weight": synth_tensor(0, TID_EMBED, V, H, 0.02), "model.norm.weight": np.ones(H, np.float32)}
    wts["lm_head.weight"] = wts["model.embed_tokens.weight"]
    for l in range(sample_layers):
        p = f"model.layers.{l}."
        t = lambda k: layer_tensor_id(l, k)  # noqa: E731
        for key, kind, shape in (("self_attn.q_proj.weight", "q", (nq * hd, H)), ("self_attn.k_proj.weight", "k", (nkv * hd, H)),
                                 ("self_attn.v_proj.weight", "v", (nkv * hd, H)), ("self_attn.o_proj.weight", "o", (H, nq * hd)),
                                 ("mlp.gate_proj.weight", "gate", (I, H)), ("mlp.up_proj.weight", "up", (I, H)),
                                 ("mlp.down_proj.weight", "down", (H, I))):
            wts[p + key] = synth_tensor(0, t(kind), shape[0], shape[1], 0.02)
        for key in ("input_layernorm.weight", "post_attention_layernorm.weight"):
            wts[p + key] = np.ones(H, np.float32)
        wts[p + "self_attn.q_norm.weight"] = np.ones(hd, np.float32)
        wts[p + "self_attn.k_norm.weight"] = np.ones(hd, np.float32)
    cache = {k: np.asarray(v, dtype=np.float64) for k, v in wts.items()}
    prompt = [int(t) for t in np.random.default_rng(0).integers(0, 151643, size=w["prompt"])]
    window = prompt + [cfg["mask_token_id"]] * w["block"]
    frontier = list(range(w["prompt"], w["prompt"] + w["block"]))
    t0 = time.perf_counter()
    logits = ofwd.forward_fp64(wts, sub, window, prompt_len=0, block_size=w["block"], output_rows=frontier,
                               cast=lambda k: cache.get(k))
    t_fwd = time.perf_counter() - t0
    t1 = time.perf_counter()
    osel.max_prob_rows(logits.astype(np.float32))
    t_sel = time.perf_counter() - t1
    # lm_head + selector are inside t_fwd / t_sel; scale the transformer layers to the full depth.
    t_head = t_fwd  # measured below with zero layers to split layer cost from the head
    t2 = time.perf_counter()
    ofwd.forward_fp64(wts, dict(cfg, layer_count=0), window, prompt_len=0, block_size=w["block"],
                      output_rows=frontier, cast=lambda k: cache.get(k))
    t_head = time.perf_counter() - t2
    per_layer = max(0.0, t_fwd - t_head) / sample_layers
    step_s = t_head + per_layer * L + t_sel
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    return {"ms_per_denoising_step": step_s * 1e3, "step_s": step_s, "cores": cores,
            "sample": (f"one {args.workload} denoising step (window {len(window)} rows, float64 spec forward; "
                       f"{sample_layers} of {L} layers timed and scaled to {L}, plus lm_head and selector on "
                       f"{w['block']} frontier rows); measured {t_fwd + t_sel + t_head:.1f} s")}


SEL_V = 151936
SEL_SHAPES = [(1, 32), (1, 256), (8, 32), (8, 256)]


def _selector_case(B: int, L: int, seed: int, device):
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    logits = torch.randn(B * L, SEL_V, generator=g, device=device, dtype=torch.float32) * 3.0
    mask = torch.rand(B, L, generator=g, device=device) < 0.5
    rows = torch.nonzero(mask.reshape(-1)).reshape(-1).to(torch.int32)
    counts = mask.sum(1).tolist()
    offsets = torch.tensor(np.concatenate([[0], np.cumsum(counts)]), dtype=torch.int32, device=device)
    return logits, mask, rows, offsets


def _run_selector(args, world, rank, local) -> dict | None:
    """cfg4: selector + choices over the masked rows; CUDA-event time per step, L2 flushed between
    steps (a 256 MB write) so every variant reads its logits from HBM."""
    import torch

    from diffusorrt_b200 import _lib, build, kernels

    if rank == 0:
        build.build()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        build.build()
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    variants = {}
    launches = 0
    headline = None
    clocks = ClockSampler(local)
    clocks.__enter__()
    for B, L in SEL_SHAPES:
        logits, mask, rows, offsets = _selector_case(B, L, 1000 * B + L + rank, dev)
        n = rows.numel()
        scratch = kernels.selector_scratch(n, SEL_V, dev)
        conf = torch.empty(n, dtype=torch.float64, device=dev)
        tok = torch.empty(n, dtype=torch.int32, device=dev)
        chosen = torch.empty(n, dtype=torch.int32, device=dev)
        tie = torch.empty(B, dtype=torch.int32, device=dev)
        for mode_name, mode in (("max_prob", _lib.SELECT_MAX_PROB), ("entropy", _lib.SELECT_NEG_ENTROPY)):
            def step():
                kernels.select_gather(logits, rows, mode=mode, temperature=1.0, scratch=scratch, conf=conf, token=tok)
                for k in (1, 4, 8):
                    kernels.select_choices(conf, offsets, mode=kernels.CHOICE_TOPK, k=k, chosen=chosen, tie=tie)
                kernels.select_choices(conf, offsets, mode=kernels.CHOICE_THRESHOLD, tau=0.9, chosen=chosen, tie=tie)
            for _ in range(args.warmup):
                step()
            torch.cuda.synchronize()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
            for e0, e1 in ev:
                flush.fill_(1)
                e0.record()
                step()
                e1.record()
            torch.cuda.synchronize()
            ms = float(np.mean([e0.elapsed_time(e1) for e0, e1 in ev]))
            alg = n * SEL_V * 4
            gbs = alg / (ms * 1e-3) / 1e9
            launches += args.steps * (5 + (1 if mode == _lib.SELECT_NEG_ENTROPY else 0))
            variants[f"B{B}_L{L}_{mode_name}"] = {"masked_rows": n, "us_per_step": round(ms * 1e3, 2),
                                                   "GB_per_s": round(gbs, 1)}
            if (B, L, mode_name) == (8, 256, "max_prob"):
                headline = (ms, alg, n, logits, rows, offsets, mask)
    clocks.__exit__(None, None, None)
    ms, alg, n, logits, rows, offsets, mask = headline
    # End to end through the C ABI from pinned host memory: the [B, L, V] logits and the masked-row
    # list go up, the choices come back.
    host_logits = logits.cpu().pin_memory()
    host_rows = rows.cpu().pin_memory()
    host_off = offsets.cpu().pin_memory()
    d_logits = torch.empty_like(logits)
    d_rows = torch.empty_like(rows)
    d_off = torch.empty_like(offsets)
    scratch = kernels.selector_scratch(n, SEL_V, dev)
    conf = torch.empty(n, dtype=torch.float64, device=dev)
    tok = torch.empty(n, dtype=torch.int32, device=dev)
    chosen = torch.empty(n, dtype=torch.int32, device=dev)
    tie = torch.empty(8, dtype=torch.int32, device=dev)
    host_chosen = torch.empty(n, dtype=torch.int32).pin_memory()
    e2e = []
    for i in range(args.warmup + args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        d_logits.copy_(host_logits, non_blocking=True)
        d_rows.copy_(host_rows, non_blocking=True)
        d_off.copy_(host_off, non_blocking=True)
        kernels.select_gather(d_logits, d_rows, mode=_lib.SELECT_MAX_PROB, scratch=scratch, conf=conf, token=tok)
        kernels.select_choices(conf, d_off, mode=kernels.CHOICE_TOPK, k=1, chosen=chosen, tie=tie)
        host_chosen.copy_(chosen, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        if i >= args.warmup:
            e2e.append(e0.elapsed_time(e1))
    e2e_ms = float(np.mean(e2e))
    if rank != 0:
        return None
    peaks = _peaks()
    gbs = alg / (ms * 1e-3) / 1e9
    return {
        "metric": "unmask selector throughput (cfg4: fp32 [B, L, 151936] logits, 50% masked, softmax confidence + "
                  "top-k/threshold choices)",
        "value": round(world * gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0, 3^2) logits, Bernoulli(0.5) mask)",
        "config": {"workload": "cfg4: B 8, L 256, V 151936, max-prob, top-k 1/4/8 + threshold 0.9 per step",
                   "masked_rows": n, "l2": "flushed before every timed step (256 MB write)", "variants": variants},
        "roofline": {"bound": "hbm", "kernel": "sel_pass1_kernel + sel_choose_kernel (one step)",
                     "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(gbs / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                     "algorithmic_bytes_per_step": int(alg), "traffic": None},
        "e2e": {"value": round(world * alg / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": int(logits.numel() * 4 + rows.numel() * 4 + offsets.numel() * 4),
                "d2h_bytes_per_step": int(n * 4)},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
    }


def _cpu_selector_baseline(sample_rows: int = 48) -> dict:
    """The reference selector restated (float64 NumPy, one thread) on a sample of cfg4 rows."""
    from oracle import selector as osel

    rng = np.random.default_rng(7)
    rows = (rng.standard_normal((sample_rows, SEL_V), dtype=np.float32) * np.float32(3.0)).astype(np.float32)
    t0 = time.perf_counter()
    conf, _ = osel.max_prob_rows(rows)
    for k in (1, 4, 8):
        osel.topk_choices(conf, k)
    osel.threshold_choices(conf, 0.9)
    dt = time.perf_counter() - t0
    return {"GB_per_s": sample_rows * SEL_V * 4 / dt / 1e9, "seconds": dt,
            "sample": f"{sample_rows} rows of 151936 fp32 logits: max-prob confidence, top-k 1/4/8 and threshold choices"}


def _profile_case(args) -> None:
    """A small, self-contained decode run for profilers (``--profile-case``): the bench workload's
    kernels at the bench's shapes with few launches before them, about 2 GB on the device.

      cfg1:  Qwen3-0.6B-architecture BD3LM, one --pc-prompt (4096) token prompt and one --pc-gen (32)
             token block under block_threshold with --pc-rounds (8) rounds;
      quant: the 4-bit affine model under bd3_fixed_quota, 16 rounds per 32-token block;
             every forward, prompt chunks included, runs the quantized decode linear in 64-row chunks;
             --pc-bits 8 loads the int8 weight-only model instead;
      cfg1 with --pc-temperature T > 0: bd3_fixed_quota with 16 rounds per block, each row's token
             drawn by the sampling selector (Gumbel keys, seed 0);
      dream: Dream-7B full canvas (prompt 256 + canvas 256), entropy_count over --pc-steps (4) steps,
             --pc-layers layers (0: the model's 28); ~15 GB of synthetic weights.
      d2f:   Dream-7B on the D2F graph (prompt 256 as the mask origin), d2f_block_pipeline with the
             reference's active-window preset (block 8, tau_conf 0.8, tau_add 0.1, tau_act 0.95) over
             --pc-steps (4) denoising steps of a 256-token canvas.

    Kernel order, for a profiler's name filter and skip count: the prompt prefill launches one
    embed_rows_kernel and two rmsnorm_bf16_kernel per layer (with the prefill linears and attention);
    every denoising step then launches plan_kernel, embed_rows_kernel, per layer [rmsnorm, gemm_decode
    (QKV), attn_decode, attn_merge, gemm_decode (o), rmsnorm, gemm_decode (gate/up), gemm_decode
    (down)], then rmsnorm, gemm_lm_kernel (lm_head; gemm_decode for the 4-bit model), sel_pass1_kernel
    and commit_kernel. A Dream step: dream_plan_kernel, embed_rows_kernel, per layer [rmsnorm,
    gemm_swapab (QKV), attention, gemm_swapab (o), rmsnorm, gemm_swapab (gate/up), gemm_swapab
    (down)], rmsnorm, gemm_swapab (lm_head), sel_topp_entropy_kernel, dream_commit_kernel.

    Prints one JSON line: denoising steps run, kernel launches of the request and ms per step."""
    if args.profile_case == "d2f":
        from diffusorrt_b200 import Runtime
        from diffusorrt_b200.config import DREAM_7B

        rt = Runtime(model_config=dict(DREAM_7B), synthetic_seed=0, device_ordinal=0, max_seq=512, max_prefill_rows=256)
        sess = rt.session({"decode_strategy": "d2f_block_pipeline", "block_size": 8})
        prompt = [int(t) for t in np.random.default_rng(0).integers(0, 151643, size=256)]
        res = sess.generate(prompt, max_tokens=256, steps=args.pc_steps, block_size=8, decode_strategy="d2f_block_pipeline",
                            confidence_threshold=0.8, add_threshold=0.1, activate_threshold=0.95, mask_origin="prompt")
        forwards = int(res["forward_count"])
        print(json.dumps({"prompt": 256, "gen": 256, "forwards": forwards, "kernel_launches": int(res["kernel_launches"]),
                          "decode_ms_per_step": res["decode_ms"] / max(1, forwards)}), flush=True)
        sess.close()
        rt.close()
        return
    args.dream = args.profile_case == "dream"
    args.quant = args.profile_case == "quant"
    args.prompt, args.gen, args.rounds, args.steps, args.layers = (args.pc_prompt, args.pc_gen, args.pc_rounds,
                                                                    args.pc_steps, args.pc_layers)
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
    engine = {"linear_quant_bits": args.pc_bits, "linear_quant_group_size": 64} if args.quant else None
    rt = Runtime(model_config=cfg, synthetic_seed=0, device_ordinal=0, max_seq=max_seq,
                 max_prefill_rows=min(4096, ((args.prompt + 127) // 128) * 128), engine_config=engine)
    fixed = args.quant or args.pc_temperature > 0
    strategy = "bd3_fixed_quota" if fixed else "block_threshold"
    sess = rt.session({"decode_strategy": strategy, "block_size": 32})
    prompt = [int(t) for t in np.random.default_rng(0).integers(0, 151643, size=args.prompt)]
    steps = (args.gen // 32) * (16 if fixed else args.rounds)
    res = sess.generate(prompt, max_tokens=args.gen, steps=steps, block_size=32, decode_strategy=strategy,
                        confidence_threshold=0.9, rounds_per_block=0 if fixed else args.rounds,
                        temperature=args.pc_temperature)
    forwards = int(res["forward_count"])
    print(json.dumps({"prompt": args.prompt, "gen": args.gen, "forwards": forwards,
                      "kernel_launches": int(res["kernel_launches"]),
                      "decode_ms_per_step": res["decode_ms"] / max(1, forwards)}), flush=True)
    sess.close()
    rt.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="cfg1", choices=sorted(WORKLOADS) + ["cfg2", "cfg4"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-case", choices=["cfg1", "quant", "dream", "d2f"],
                    help="run one small decode for a profiler instead of the benchmark (see _profile_case)")
    ap.add_argument("--pc-prompt", type=int, default=4096)
    ap.add_argument("--pc-gen", type=int, default=32)
    ap.add_argument("--pc-rounds", type=int, default=8)
    ap.add_argument("--pc-steps", type=int, default=4)
    ap.add_argument("--pc-layers", type=int, default=0)
    ap.add_argument("--pc-bits", type=int, default=4, choices=(4, 8), help="--profile-case quant: weight bits")
    ap.add_argument("--pc-temperature", type=float, default=0.0,
                    help="--profile-case cfg1: > 0 samples each row's token (bd3_fixed_quota)")
    args = ap.parse_args()
    if args.profile_case:
        _profile_case(args)
        return
    args.warmup = max(3, args.warmup)
    world, rank, local = _dist()
    if args.impl == "reference" and args.workload == "cfg4":
        if rank != 0:
            return
        samples = [_cpu_selector_baseline() for _ in range(max(1, min(args.steps, 3)))]
        gbs = float(np.mean([x["GB_per_s"] for x in samples]))
        cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
        print(json.dumps({"metric": "unmask selector throughput (cfg4)", "impl": "reference", "value": round(gbs, 3),
                          "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
                          "data": "synthetic", "config": {"workload": "cfg4"},
                          "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": 1, "kind": "port",
                                           "sample": samples[0]["sample"]},
                          "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return
    if args.impl == "reference" and args.workload == "cfg2":
        if rank != 0:
            return
        cb = _cpu_dream_baseline()
        tokens = DREAM["gen"]
        sched_steps = DREAM["steps"]
        value = tokens / (cb["step_s"] * sched_steps)
        print(json.dumps({"metric": METRIC, "impl": "reference", "value": value, "unit": "tokens/s", "n_gpus": world,
                          "steps": args.steps, "warmup": args.warmup, "ms_per_step": cb["step_s"] * sched_steps * 1e3,
                          "ms_per_denoising_step": cb["ms_per_denoising_step"], "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
                          "config": {"workload": "cfg2", "prompt": DREAM["prompt"], "gen": DREAM["gen"]},
                          "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cb["cores"], "kind": "port",
                                           "sample": cb["sample"]},
                          "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return
    if args.impl == "reference":
        if rank != 0:
            return
        w = WORKLOADS[args.workload]
        if w.get("model") == "dream":
            print(json.dumps({"impl": "reference", "unavailable": "the d2f workload's CPU reference step is cfg2's "
                              "(same Dream-7B model): run --impl reference --workload cfg2"}), flush=True)
            return
        samples = [_cpu_baseline(args) for _ in range(max(1, min(args.steps, 2)))]
        step_s = float(np.mean([s["step_s"] for s in samples]))
        steps_per_request = 16 * 8 if args.workload == "cfg1" else 128
        tokens_per_request = {"cfg1": 16 * 8, "cfg3": 256}.get(args.workload, 128)
        value = tokens_per_request / (step_s * steps_per_request)
        line = {"metric": METRIC, "impl": "reference", "value": value, "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * steps_per_request * 1e3,
                "ms_per_denoising_step": step_s * 1e3, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f64", "data": "synthetic",
                "config": {"workload": args.workload, "prompt": w["prompt"], "gen": w["gen"]},
                "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": samples[0]["cores"], "kind": "port",
                                 "sample": samples[0]["sample"]},
                "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        from datetime import timedelta

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device(f"cuda:{local}"))
    if args.workload == "cfg4":
        line = _run_selector(args, world, rank, local)
        if rank == 0 and line is not None:
            if not args.no_cpu_baseline and world == 1:
                cb = _cpu_selector_baseline()
                line["cpu_baseline"] = {"value": round(cb["GB_per_s"], 3), "unit": "GB/s", "cores": 1, "kind": "port",
                                        "sample": cb["sample"]}
            print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    if args.workload == "cfg2":
        line = _run_dream(args, world, rank, local)
        if rank == 0 and line is not None:
            if not args.no_cpu_baseline and world == 1:
                cb = _cpu_dream_baseline()
                steps = line["config"]["denoising_steps_per_request"]
                tokens = line["config"]["committed_tokens_per_request"]
                line["cpu_baseline"] = {"value": round(tokens / (cb["step_s"] * steps), 6), "unit": "tokens/s",
                                        "cores": cb["cores"], "kind": "port", "sample": cb["sample"],
                                        "ms_per_denoising_step": round(cb["ms_per_denoising_step"], 1)}
            print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    line = _run_ours(args, world, rank, local)
    if rank == 0 and line is not None:
        # (the d2f workload's model is cfg2's: its CPU baseline is cfg2's line)
        if not args.no_cpu_baseline and world == 1 and WORKLOADS[args.workload].get("model") != "dream":
            cb = _cpu_baseline(args)
            steps = line["config"]["denoising_steps_per_request"]
            tokens = line["config"]["committed_tokens_per_request"]
            line["cpu_baseline"] = {"value": round(tokens / (cb["step_s"] * steps), 6), "unit": "tokens/s",
                                    "cores": cb["cores"], "kind": "port", "sample": cb["sample"],
                                    "ms_per_denoising_step": round(cb["ms_per_denoising_step"], 1)}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
