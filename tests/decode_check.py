"""Whole-decode check of a device BD3 trajectory against the oracle, step by step.

A random-init model's decode is decided by confidence gaps far below the bf16 forward error (at
Qwen3-0.6B geometry half of the frontier rows' confidences lie within 2e-4 of each other, against
a logit tolerance of about 0.03 of the logit scale), so no independent implementation — the
reference's MLX on another device included — reproduces its trajectory bit for bit. The check is
therefore made along the device's own trajectory: before every step the oracle (the reference's
MLX-contract forward, prefix-K/V cached) scores the frontier on the device's canvas, and the
device's step must be the oracle's step up to the stated logit tolerance E (bf16_tolerance: at
most MAX_FACTOR u of the logit RMS per logit):

* every frontier row's confidence: |log conf_dev - log conf_oracle| <= 2 E (the max-prob confidence
  is exp(x_max - logsumexp x), and each of the two terms moves by at most E);
* the chosen rows: no unchosen row's oracle log-confidence exceeds a chosen row's by more than 4 E;
* each committed token's oracle logit is within 2 E of its row's oracle maximum.

Steps where the device's choice and tokens equal the oracle's exactly are counted and reported.
"""
from __future__ import annotations

import numpy as np

from bf16_tolerance import MAX_FACTOR, U_BF16
from oracle import forward as ofwd
from oracle import policy as opol
from oracle import selector as osel


def check_bd3_trajectory(dev: dict, weights: dict, cfg: dict, prompt: list[int], *, gen: int, steps: int,
                         block_size: int, quant: dict | None = None, quant_bits: int = 4) -> dict:
    mask, eos = cfg["mask_token_id"], cfg["eos_token_id"]
    c = opol.Canvas(list(prompt) + [mask] * gen, len(prompt), mask, eos)
    pol = opol.BD3FixedQuota(block_size=block_size, steps=steps, prompt_len=len(prompt), gen_len=gen)
    cache = ofwd.PrefixKV(cfg)
    rope = ofwd.rope_half_tables(len(c.x), cfg["head_dim"], float(cfg["rope_theta"]))
    exact = 0
    worst = {"conf": 0.0, "rows": 0.0, "token": 0.0}
    trace = iter(dev["trace"])
    forwards = 0
    for step in range(pol.iteration_limit):
        plan = pol.plan(c, step)
        if plan.action == "stop":
            break
        if plan.action == "skip":
            continue
        tr = next(trace)
        forwards += 1
        assert tr["step"] == step and tr["frontier"] == plan.frontier, step
        frozen = (min(plan.frontier) // block_size) * block_size
        logits = ofwd.forward_mlx_cached(weights, cfg, c.x[:plan.window_end], cache, frozen=frozen,
                                         output_rows=plan.frontier, rope=rope, quant=quant, quant_bits=quant_bits)
        conf, tok = osel.max_prob_rows(logits)
        E = MAX_FACTOR * U_BF16 * float(np.sqrt(np.mean(np.square(logits.astype(np.float64)))))
        lc_dev, lc_or = np.log(np.asarray(tr["scores"])), np.log(conf)
        d_conf = float(np.abs(lc_dev - lc_or).max())
        assert d_conf <= 2 * E, (step, d_conf, E)
        chosen = tr["chosen"]
        others = [r for r in range(len(plan.frontier)) if r not in chosen]
        d_rows = float(max(lc_or[others]) - min(lc_or[chosen])) if others else -np.inf
        assert d_rows <= 4 * E, (step, d_rows, E)
        for r in chosen:
            d_tok = float(logits[r].max() - logits[r][tr["tokens"][r]])
            assert d_tok <= 2 * E, (step, r, d_tok, E)
            worst["token"] = max(worst["token"], d_tok / E)
        worst["conf"] = max(worst["conf"], d_conf / E)
        worst["rows"] = max(worst["rows"], d_rows / E)
        if sorted(pol.select(conf)) == chosen and all(tr["tokens"][r] == tok[r] for r in chosen):
            exact += 1
        for r in chosen:  # follow the device's commits
            c.x[plan.frontier[r]] = tr["tokens"][r]
    assert forwards == dev["forward_count"]
    assert c.x == dev["x"]
    return {"steps": forwards, "exact_steps": exact, "worst_over_E": worst}
