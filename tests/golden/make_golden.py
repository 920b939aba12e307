"""Generate the golden vectors that pin the oracle to the reference implementation.

Runs the reference's own CPU code (importable without MLX) on seeded inputs and writes small
fixtures next to this script. The reference tree is only read; nothing here runs on the GPU
box (the fixtures travel, this script does not need to).

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference /path/to/reference

Fixtures:
  selector.npz   max-prob / entropy (incl. temperature + top-p) / top-k / threshold / MASK exclusion
  decode.json    BD3 fixed-quota, block-threshold and entropy-count decode trajectories under the
                 deterministic stand-in forward of fake_forward.py
  forward.npz    float64 executable-spec logits of a tiny synthetic model, d2f_hybrid and bidirectional
  tables.npz     float32 RoPE rows and d2f_hybrid visibility matrices
  cases.json     the reference BD3 window cases (model_coverage qwen3_06b_bd3lm_v0_1) + ABI constants
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))

from fake_forward import fake_logits  # noqa: E402

TINY = dict(layer_count=2, hidden_size=128, attention_heads=4, num_kv_heads=2, head_dim=32,
            intermediate_size=256, vocab_size=320, rms_norm_eps=1e-6, rope_theta=1e6)


def _selector(dr) -> dict:
    rng = np.random.default_rng(20261201)
    out = {}
    small = rng.normal(0.0, 3.0, size=(6, 4096)).astype(np.float32)
    small[3, 100] = small[3, 2000] = np.float32(small[3].max() + 1.0)  # exact tie on the max
    wide = rng.normal(0.0, 3.0, size=(1, 151936)).astype(np.float32)
    sharp = (rng.normal(0.0, 1.0, size=(5, 1024)) * 12.0).astype(np.float32)
    for name, arr in (("small", small), ("wide", wide), ("sharp", sharp)):
        out[f"{name}_logits"] = arr
        conf, tok = dr._raw_max_prob_rows_exact(arr)
        out[f"{name}_maxprob_conf"] = np.asarray(conf, dtype=np.float64)
        out[f"{name}_maxprob_tok"] = np.asarray(tok, dtype=np.int64)
        for tag, temp, top_p in (("t1", 1.0, None), ("t02p095", 0.2, 0.95)):
            conf, tok = dr._entropy_confidence(arr, temperature=temp, top_p=top_p)
            out[f"{name}_ent_{tag}_conf"] = np.asarray(conf, dtype=np.float32)
            out[f"{name}_ent_{tag}_tok"] = np.asarray(tok, dtype=np.int64)
    # Temperature sampling (TopConfidence at T > 0): tokens and raw probabilities of the draws.
    srng = np.random.default_rng(20261202)
    for name, arr in (("small", small), ("wide", wide), ("sharp", sharp)):
        positions = [int(p) for p in srng.integers(0, 5000, size=arr.shape[0])]
        out[f"{name}_sample_pos"] = np.asarray(positions, dtype=np.int64)
        for tag, temp, seed, fwd in (("a", 0.7, 11, 0), ("b", 2.0, 2**63 + 3, 17)):
            conf, tok = dr._sampled_max_prob_confidence(arr, temperature=temp, seed=seed, step=fwd, positions=positions)
            out[f"{name}_sample_{tag}_conf"] = np.asarray(conf, dtype=np.float64)
            out[f"{name}_sample_{tag}_tok"] = np.asarray(tok, dtype=np.int64)
            out[f"{name}_sample_{tag}_args"] = np.asarray([temp, float(seed), float(fwd)], dtype=np.float64)
            out[f"{name}_sample_{tag}_seed"] = np.asarray([seed], dtype=np.uint64)
    out["noise_row"] = np.asarray(dr.sampling_noise(5, 2, 40, 4096), dtype=np.float32)
    excl = dr._exclude_mask_token(small[:2], mask_token_id=7)
    out["excl_logits"] = np.asarray(excl, dtype=np.float32)
    confs = rng.random(size=(4, 32))
    confs[1, 5] = confs[1, 9] = 0.95  # tie
    confs[2, :] = rng.random(32) * 0.5  # nothing clears 0.9
    confs[3, 3] = 0.9  # exactly on the threshold
    out["choice_conf"] = confs
    for k in (1, 4, 8):
        out[f"choice_topk{k}"] = np.asarray([dr._topk_count_choices(c, transfer_count=k) for c in confs], dtype=np.int64)
    thr = [dr._threshold_choices(c, threshold=0.9) for c in confs]
    out["choice_thr_flat"] = np.asarray([i for t in thr for i in t], dtype=np.int64)
    out["choice_thr_len"] = np.asarray([len(t) for t in thr], dtype=np.int64)
    return out


def _decode(ds) -> dict:
    traces = {}

    def run(name, strategy, *, prompt_len, gen, steps, block_size, vocab, mask, eos, scale, **opts):
        prompt = [int(t) for t in np.random.default_rng(prompt_len * 7 + gen).integers(0, mask, size=prompt_len)]
        calls = []

        def forward(ids):
            calls.append(list(ids))
            return fake_logits(ids, vocab, scale=scale)

        decode = ds.DecodeRequest(decode_strategy=strategy, steps=steps, block_size=block_size, **opts).prepare(
            prefix_token_ids=prompt, token_count=gen, mask_token_id=mask, eos_token_id=eos)
        res = decode.run(forward_fn=forward)
        traces[name] = dict(
            strategy=strategy, prompt=prompt, gen=gen, steps=steps, block_size=block_size, vocab=vocab,
            mask=mask, eos=eos, scale=scale, options=opts, final=list(decode.state.x),
            forward_count=res.forward_count, committed_token_count=res.committed_token_count,
            iteration_count=res.iteration_count, finish_reason=res.finish_reason,
            remaining_mask_count=res.remaining_mask_count, visible=list(res.visible_generated_token_ids),
            window_lengths=[len(c) for c in calls])

    run("bd3_cfg0_shape", "bd3_fixed_quota", prompt_len=64, gen=128, steps=128, block_size=32, vocab=512,
        mask=500, eos=501, scale=3.0)
    run("bd3_k2", "bd3_fixed_quota", prompt_len=32, gen=96, steps=48, block_size=32, vocab=512,
        mask=500, eos=501, scale=3.0)
    run("bd3_ragged_quota", "bd3_fixed_quota", prompt_len=32, gen=40, steps=10, block_size=16, vocab=256,
        mask=250, eos=251, scale=3.0)
    run("bd3_eos", "bd3_fixed_quota", prompt_len=32, gen=128, steps=64, block_size=32, vocab=64,
        mask=60, eos=3, scale=3.0)
    run("bd3_sampled", "bd3_fixed_quota", prompt_len=32, gen=64, steps=32, block_size=32, vocab=512,
        mask=500, eos=501, scale=3.0, temperature=0.8, seed=1234)
    run("block_threshold", "block_threshold", prompt_len=32, gen=96, steps=200, block_size=32, vocab=512,
        mask=500, eos=501, scale=6.0, confidence_threshold=0.9)
    # d2f_block_pipeline: blocks of 8 with the product preset's thresholds; scale 6 gives rows that
    # clear tau_conf and rows that do not (semi-activated blocks waiting, forced argmax commits,
    # several blocks in the window); a small vocabulary makes EOS land early in one case
    run("d2f_pipeline", "d2f_block_pipeline", prompt_len=24, gen=64, steps=200, block_size=8, vocab=512,
        mask=500, eos=501, scale=6.0, confidence_threshold=0.8, d2f_add_threshold=0.1,
        d2f_activate_threshold=0.95)
    run("d2f_pipeline_tau06", "d2f_block_pipeline", prompt_len=16, gen=60, steps=200, block_size=8, vocab=256,
        mask=250, eos=251, scale=5.0, confidence_threshold=0.6, d2f_add_threshold=0.25,
        d2f_activate_threshold=0.9)
    run("d2f_pipeline_eos", "d2f_block_pipeline", prompt_len=16, gen=64, steps=200, block_size=8, vocab=48,
        mask=40, eos=3, scale=6.0, confidence_threshold=0.8, d2f_add_threshold=0.1,
        d2f_activate_threshold=0.95)
    run("d2f_pipeline_capped", "d2f_block_pipeline", prompt_len=24, gen=64, steps=12, block_size=16, vocab=512,
        mask=500, eos=501, scale=6.0, confidence_threshold=0.9, d2f_add_threshold=0.1,
        d2f_activate_threshold=0.95)
    run("entropy_count", "entropy_count", prompt_len=16, gen=32, steps=24, block_size=8, vocab=256,
        mask=250, eos=251, scale=3.0, temperature=0.2, top_p=0.95, eps=1e-3)
    return traces


def _forward(numpyref, build_graph_ir) -> dict:
    from oracle.numerics import synth_weights

    cfg = dict(TINY, uses_qk_norm=True, uses_shifted_logits=False, bias_present=False,
               attention_mask_kind="d2f_hybrid")
    weights = synth_weights(dict(TINY, qk_norm=True, tied_lm_head=True), seed=5, linear_std=0.05, embed_std=0.5)
    graph = build_graph_ir(cfg)
    ids = [int(t) for t in np.random.default_rng(9).integers(0, TINY["vocab_size"], size=24)]
    w64 = {k: np.asarray(v, dtype=np.float64) for k, v in weights.items()}
    d2f = numpyref.interpret_graph(graph, weights=w64, token_ids=ids, mask_geometry={"prompt_len": 0, "block_size": 8})
    cfg_b = dict(cfg, attention_mask_kind="bidirectional")
    bidir = numpyref.interpret_graph(build_graph_ir(cfg_b), weights=w64, token_ids=ids)
    return {"ids": np.asarray(ids, dtype=np.int64), "d2f_logits": np.asarray(d2f), "bidir_logits": np.asarray(bidir)}


def _tables(mlx_forward, numpyref) -> dict:
    c, s = mlx_forward._rope_tables(seq_len=4608, head_dim=128, rope_theta=1e6, rope_scaling=None)
    rows = np.asarray([0, 1, 2, 31, 32, 100, 1000, 4095, 4607], dtype=np.int64)
    out = {"rope_rows": rows, "rope_cos": c[rows, 0, :64], "rope_sin": s[rows, 0, :64]}
    for name, (seq, pl, bs) in {"vis_a": (12, 0, 4), "vis_b": (13, 5, 3), "vis_c": (40, 0, 32)}.items():
        out[name] = np.asarray(numpyref.d2f_hybrid_visibility(seq, prompt_len=pl, block_size=bs))
        out[name + "_geom"] = np.asarray([seq, pl, bs])
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DIFFUSORRT_REFERENCE"),
                    help="checkout of the reference project (or set DIFFUSORRT_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference checkout with --reference or DIFFUSORRT_REFERENCE")
    sys.path.insert(0, str(Path(args.reference) / "python" / "src"))
    sys.dont_write_bytecode = True
    from edllm.abi import ABI_VERSION
    from edllm.abi import enums
    from edllm.abi.forward import AbiStatus
    from edllm.backends import decode_session as ds
    from edllm.backends import diffusion_runtime as dr
    from edllm.backends import mlx_forward
    from edllm.graph import numpyref
    from edllm.graph.emitter import build_graph_ir

    np.savez_compressed(HERE / "selector.npz", **_selector(dr))
    (HERE / "decode.json").write_text(json.dumps(_decode(ds), indent=1))
    np.savez_compressed(HERE / "forward.npz", **_forward(numpyref, build_graph_ir))
    np.savez_compressed(HERE / "tables.npz", **_tables(mlx_forward, numpyref))
    cases = json.loads((Path(args.reference) / "python/src/edllm/model_coverage/data/cases/qwen3_06b_bd3lm_v0_1.json").read_text())
    meta = {
        "cases": cases["cases"],
        "abi_version": list(ABI_VERSION),
        "abi_status": {m.name: int(m.value) for m in AbiStatus},
        "decode_strategy": {k: int(v) for k, v in enums.DECODE_STRATEGY_BY_NAME.items()},
        "commit_policy": {k: int(v) for k, v in enums.COMMIT_POLICY_BY_NAME.items()},
        "attention_mask_kind": {k: int(v) for k, v in enums.ATTENTION_MASK_KIND_BY_NAME.items()},
        "generated_with": {"numpy": np.__version__, "python": platform.python_version(), "machine": platform.machine()},
    }
    (HERE / "cases.json").write_text(json.dumps(meta, indent=1))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
