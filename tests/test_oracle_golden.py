"""The CPU oracle against golden vectors produced by the reference implementation itself
(tests/golden/make_golden.py). Bit-exact where the reference is deterministic on this host;
confidence values within a few ulp where NumPy's float64 exp may dispatch differently."""
from __future__ import annotations

import json

import numpy as np
import pytest

from fake_forward import fake_logits
from oracle import forward, policy, selector
from oracle.numerics import rope_half_tables, synth_weights


@pytest.fixture(scope="module")
def sel(golden_dir):
    return np.load(golden_dir / "selector.npz")


@pytest.mark.parametrize("name", ["small", "wide", "sharp"])
def test_max_prob_rows(sel, name):
    conf, tok = selector.max_prob_rows(sel[f"{name}_logits"])
    assert tok == list(sel[f"{name}_maxprob_tok"])
    np.testing.assert_allclose(conf, sel[f"{name}_maxprob_conf"], rtol=1e-13, atol=0)


def test_max_prob_token_is_first_max_logit(sel):
    logits = sel["small_logits"]
    _, tok = selector.max_prob_rows(logits)
    assert tok == [int(np.argmax(r)) for r in logits]
    assert tok[3] == 100  # exact tie on the max resolves to the first index


@pytest.mark.parametrize("name", ["small", "wide", "sharp"])
@pytest.mark.parametrize("tag,temp,top_p", [("t1", 1.0, None), ("t02p095", 0.2, 0.95)])
def test_neg_entropy_rows(sel, name, tag, temp, top_p):
    conf, tok = selector.neg_entropy_rows(sel[f"{name}_logits"], temperature=temp, top_p=top_p)
    assert tok == list(sel[f"{name}_ent_{tag}_tok"])
    np.testing.assert_allclose(conf, sel[f"{name}_ent_{tag}_conf"], rtol=2e-7, atol=0)


def test_exclude_mask(sel):
    np.testing.assert_array_equal(selector.exclude_mask_token(sel["small_logits"][:2], 7), sel["excl_logits"])


def test_choices(sel):
    confs = sel["choice_conf"]
    for k in (1, 4, 8):
        got = [selector.topk_choices(c, k) for c in confs]
        assert got == [list(r) for r in sel[f"choice_topk{k}"]]
    flat = [i for c in confs for i in selector.threshold_choices(c, 0.9)]
    assert flat == list(sel["choice_thr_flat"])


def _policy_for(tr):
    bs = tr["block_size"]
    if tr["strategy"] == "bd3_fixed_quota":
        pol = policy.BD3FixedQuota(block_size=bs, steps=tr["steps"], prompt_len=len(tr["prompt"]), gen_len=tr["gen"])
        return pol, pol.iteration_limit, False, "sample" if tr["options"].get("temperature", 0) > 0 else "max"
    if tr["strategy"] == "block_threshold":
        return policy.BlockThreshold(block_size=bs, threshold=tr["options"]["confidence_threshold"]), tr["steps"], True, "max"
    if tr["strategy"] == "d2f_block_pipeline":
        o = tr["options"]
        pol = policy.D2FPipeline(block_size=bs, threshold=o["confidence_threshold"], add_threshold=o["d2f_add_threshold"],
                                 activate_threshold=o["d2f_activate_threshold"])
        return pol, tr["steps"], True, "max"
    opts = tr["options"]
    return policy.EntropyCount(eps=opts["eps"], steps=tr["steps"]), tr["steps"], True, "ent"


@pytest.mark.parametrize("name", ["small", "wide", "sharp"])
@pytest.mark.parametrize("tag", ["a", "b"])
def test_sampled_rows(sel, name, tag):
    """Temperature sampling (TopConfidence at T > 0) against the reference's own draws."""
    temp, _, fwd = (float(v) for v in sel[f"{name}_sample_{tag}_args"])
    seed = int(sel[f"{name}_sample_{tag}_seed"][0])
    conf, tok, gaps = selector.sampled_max_prob_rows(sel[f"{name}_logits"], temperature=temp, seed=seed,
                                                     forward=int(fwd), positions=list(sel[f"{name}_sample_pos"]))
    assert tok == list(sel[f"{name}_sample_{tag}_tok"])
    np.testing.assert_allclose(conf, sel[f"{name}_sample_{tag}_conf"], rtol=1e-13, atol=0)
    assert np.all(gaps >= 0)


def test_sampling_noise_row(sel):
    np.testing.assert_array_equal(selector.sampling_noise(5, 2, 40, 4096), sel["noise_row"])


@pytest.mark.parametrize("name", ["bd3_cfg0_shape", "bd3_k2", "bd3_ragged_quota", "bd3_eos", "bd3_sampled",
                                  "block_threshold", "entropy_count", "d2f_pipeline", "d2f_pipeline_tau06",
                                  "d2f_pipeline_eos", "d2f_pipeline_capped"])
def test_decode_trajectory(golden_dir, name):
    tr = json.loads((golden_dir / "decode.json").read_text())[name]
    pol, limit, exclude, kind = _policy_for(tr)
    canvas = policy.Canvas(list(tr["prompt"]) + [tr["mask"]] * tr["gen"], len(tr["prompt"]), tr["mask"], tr["eos"])
    windows = []

    def score(c, frontier, window_end, step):
        ids = c.x if window_end is None else c.x[:window_end]
        windows.append(len(ids))
        rows = fake_logits(ids, tr["vocab"], scale=tr["scale"])[frontier]
        if exclude:
            rows = selector.exclude_mask_token(rows, tr["mask"])
        if kind == "max":
            return selector.max_prob_rows(rows)
        if kind == "sample":
            o = tr["options"]
            conf, tok, _ = selector.sampled_max_prob_rows(rows, temperature=o["temperature"], seed=o["seed"],
                                                          forward=len(windows) - 1, positions=frontier)
            return conf, tok
        o = tr["options"]
        return selector.neg_entropy_rows(rows, temperature=o["temperature"], top_p=o["top_p"])

    if tr["strategy"] == "block_threshold":
        # The reference block-threshold rule forwards the whole canvas.
        def score_full(c, frontier, window_end, step):
            return score(c, frontier, None, step)
        out = policy.run_loop(canvas, pol, score_full, limit)
    else:
        out = policy.run_loop(canvas, pol, score, limit)
    assert out["x"] == tr["final"]
    assert out["forward_count"] == tr["forward_count"]
    assert out["committed_token_count"] == tr["committed_token_count"]
    assert out["finish_reason"] == tr["finish_reason"]
    assert out["remaining_mask_count"] == tr["remaining_mask_count"]
    assert out["visible_token_ids"] == tr["visible"]
    assert windows == tr["window_lengths"]


def test_fp64_forward_matches_spec(golden_dir):
    g = np.load(golden_dir / "forward.npz")
    from make_golden import TINY

    w = synth_weights(dict(TINY, qk_norm=True, tied_lm_head=True), seed=5, linear_std=0.05, embed_std=0.5)
    cfg = dict(TINY)
    d2f = forward.forward_fp64(w, cfg, g["ids"], prompt_len=0, block_size=8)
    np.testing.assert_allclose(d2f, g["d2f_logits"], rtol=1e-10, atol=1e-10)
    bid = forward.forward_fp64(w, cfg, g["ids"], bidirectional=True)
    np.testing.assert_allclose(bid, g["bidir_logits"], rtol=1e-10, atol=1e-10)


def test_mlx_contract_forward_close_to_spec(golden_dir):
    """The f32/bf16 MLX-contract restatement stays within bf16 rounding of the float64 spec."""
    g = np.load(golden_dir / "forward.npz")
    from make_golden import TINY

    w = synth_weights(dict(TINY, qk_norm=True, tied_lm_head=True), seed=5, linear_std=0.05, embed_std=0.5)
    got = forward.forward_mlx(w, dict(TINY), g["ids"], prompt_len=0, block_size=8)
    ref = g["d2f_logits"]
    scale = np.abs(ref).max()
    assert np.abs(got - ref).max() <= 0.03 * scale
    assert np.mean(np.argmax(got, -1) == np.argmax(ref, -1)) >= 0.9


def test_rope_tables_and_visibility(golden_dir):
    t = np.load(golden_dir / "tables.npz")
    cos, sin = rope_half_tables(4608, 128, 1e6)
    np.testing.assert_array_equal(cos[t["rope_rows"]], t["rope_cos"])
    np.testing.assert_array_equal(sin[t["rope_rows"]], t["rope_sin"])
    for name in ("vis_a", "vis_b", "vis_c"):
        seq, pl, bs = (int(v) for v in t[name + "_geom"])
        got = forward.visible_mask(np.arange(seq), seq, prompt_len=pl, block_size=bs, bidirectional=False)
        np.testing.assert_array_equal(got, t[name])


def test_product_rope_tables_match_reference(golden_dir):
    from diffusorrt_b200.config import rope_half_tables as product_tables

    t = np.load(golden_dir / "tables.npz")
    cos, sin = product_tables(4608, 128, 1e6)
    np.testing.assert_array_equal(cos[t["rope_rows"]], t["rope_cos"])
    np.testing.assert_array_equal(sin[t["rope_rows"]], t["rope_sin"])
