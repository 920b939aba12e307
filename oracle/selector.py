"""Unmask scoring and choice rules, restated in NumPy (test infrastructure).

Each function restates one reference function of
``python/src/edllm/backends/diffusion_runtime.py`` with the same float64 operation order, so
that on the same host it reproduces the reference's values bit for bit (pinned by
``tests/test_oracle_golden.py`` against vectors the reference produced).
"""
from __future__ import annotations

import numpy as np


def max_prob_rows(logits) -> tuple[np.ndarray, list[int]]:
    """Raw-softmax top-1 probability and argmax per row (``_raw_max_prob_rows_exact``, :179-192).

    float64 copy of the f32 rows, minus the row max, exp in place, divided by the row sum;
    the confidence is the largest probability and the token its first index.
    """
    work = np.array(logits, dtype=np.float64, copy=True)
    if work.ndim != 2:
        raise ValueError("logits must be [rows, vocab]")
    work -= work.max(axis=-1, keepdims=True)
    np.exp(work, out=work)
    work /= work.sum(axis=-1, keepdims=True)
    return work.max(axis=-1), [int(t) for t in work.argmax(axis=-1)]


def _softmax64(values: np.ndarray) -> np.ndarray:
    shifted = values - values.max(axis=-1, keepdims=True)
    e = np.exp(shifted)
    return e / e.sum(axis=-1, keepdims=True)


def top_p_filter(values: np.ndarray, top_p: float) -> np.ndarray:
    """Nucleus filter (``_top_p_filter``, :358-370): sort descending (NumPy's default, unstable
    sort), drop entries whose cumulative probability exceeds top_p except the first, restore
    the original order with -inf in the dropped slots."""
    order = np.argsort(-values, axis=-1)
    ranked = np.take_along_axis(values, order, axis=-1)
    cum = np.cumsum(_softmax64(ranked), axis=-1)
    drop = cum > top_p
    drop[..., 0] = False
    kept = np.where(drop, -np.inf, ranked)
    out = np.full_like(values, -np.inf)
    np.put_along_axis(out, order, kept, axis=-1)
    return out


def neg_entropy_rows(logits, *, temperature: float, top_p: float | None) -> tuple[np.ndarray, list[int]]:
    """Negative entropy confidence and argmax token (``_entropy_confidence``, :90-114).

    float64 logits / T (T > 0), optional top-p filter, softmax, argmax; confidence
    sum(p * log(p + 1e-10)) cast to float32.
    """
    adj = np.asarray(logits, dtype=np.float64)
    if temperature > 0:
        adj = adj / float(temperature)
    if top_p is not None and top_p < 1.0:
        adj = top_p_filter(adj, float(top_p))
    probs = _softmax64(adj)
    tokens = probs.argmax(axis=-1).astype(np.int64)
    conf = np.sum(probs * np.log(probs + 1e-10), axis=-1)
    return conf.astype(np.float32), [int(t) for t in tokens]


def exclude_mask_token(logits, mask_token_id: int) -> np.ndarray:
    """MASK column to -inf for in-vocabulary sentinels (``_exclude_mask_token``, :256-282)."""
    values = np.asarray(logits, dtype=np.float32)
    if values.ndim != 2:
        raise ValueError("decode frontier logits must be rank 2")
    if not 0 <= int(mask_token_id) < values.shape[1]:
        return values
    if values.shape[1] < 2:
        raise ValueError("the mask token is the only token in the model vocabulary")
    out = values.copy()
    out[:, int(mask_token_id)] = -np.inf
    return out


def topk_choices(confidence, k: int) -> list[int]:
    """First k rows of NumPy's default (unstable) argsort of -confidence (``_topk_count_choices``,
    :290-299)."""
    return [int(i) for i in np.argsort(-np.asarray(confidence))[:k]]


def threshold_choices(confidence, tau: float) -> list[int]:
    """Rows with confidence >= tau, else the first argmax (``_threshold_choices``, :302-314)."""
    c = np.asarray(confidence, dtype=np.float64)
    hit = np.flatnonzero(c >= float(tau))
    if hit.size == 0:
        return [int(np.argmax(c))]
    return [int(i) for i in hit]


def topk_set_certified(confidence, k: int, rel: float) -> tuple[set[int], bool]:
    """The top-k set by descending confidence (lowest index first among equals) and whether
    the cut between rank k and k+1 is wider than ``rel`` relative (no near or exact tie)."""
    c = np.asarray(confidence, dtype=np.float64)
    order = sorted(range(len(c)), key=lambda i: (-c[i], i))
    chosen = set(order[:k])
    if k <= 0 or k >= len(c):
        return chosen, True
    a, b = c[order[k - 1]], c[order[k]]
    return chosen, bool(a - b > rel * abs(a))


def threshold_set_certified(confidence, tau: float, rel: float) -> tuple[set[int], bool]:
    c = np.asarray(confidence, dtype=np.float64)
    chosen = set(threshold_choices(c, tau))
    ok = bool(np.all(np.abs(c - tau) > rel * abs(tau)))
    if not np.any(c >= tau) and len(c) > 1:
        top = np.sort(c)[::-1]
        ok = ok and bool(top[0] - top[1] > rel * abs(top[0]))
    return chosen, ok


_SAMPLE_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _splitmix_mix(z):
    z = (z ^ (z >> np.uint64(30))) * _M1
    z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def sampling_noise(seed: int, forward: int, position: int, vocab: int) -> np.ndarray:
    """float32 Gumbel noise of one row (``sampling_noise``, diffusion_runtime.py:218-231): a
    splitmix64 key chained over (seed, forward + 1, position + 1), one more mix per token id + 1,
    u = (top 23 bits + 1/2) * 2^-23, g = -log(-log u) in float32."""
    with np.errstate(over="ignore"):
        key = _splitmix_mix(np.uint64(int(seed) & 0xFFFFFFFFFFFFFFFF) + _SAMPLE_GOLDEN)
        key = _splitmix_mix(key + np.uint64((int(forward) + 1) & 0xFFFFFFFFFFFFFFFF) * _SAMPLE_GOLDEN)
        key = _splitmix_mix(key + np.uint64((int(position) + 1) & 0xFFFFFFFFFFFFFFFF) * _SAMPLE_GOLDEN)
        bits = _splitmix_mix(key + np.arange(1, vocab + 1, dtype=np.uint64) * _SAMPLE_GOLDEN)
    u = ((bits >> np.uint64(41)).astype(np.float32) + np.float32(0.5)) * np.float32(2.0 ** -23)
    return -np.log(-np.log(u))


def sampled_max_prob_rows(logits, *, temperature: float, seed: int, forward: int, positions):
    """Sampled token and its raw probability per row (``_sampled_max_prob_confidence``,
    diffusion_runtime.py:234-253): token = first argmax of f64(x) + T * f64(g) (product and sum
    rounded separately), confidence = exp(x_tok - max) / sum(exp(x - max)) in float64.
    Also returns each row's gap between the two best keys (the draw's certification margin)."""
    rows = np.asarray(logits, dtype=np.float32)
    if rows.ndim != 2 or len(positions) != rows.shape[0]:
        raise ValueError("sampling needs one position per logits row")
    scores = np.empty(rows.shape[0], dtype=np.float64)
    gaps = np.empty(rows.shape[0], dtype=np.float64)
    tokens = []
    for r, pos in enumerate(positions):
        values = rows[r].astype(np.float64)
        keys = values + float(temperature) * sampling_noise(seed, forward, int(pos), rows.shape[1]).astype(np.float64)
        tok = int(np.argmax(keys))
        top2 = np.partition(keys, -2)[-2:] if keys.size > 1 else np.array([-np.inf, keys[0]])
        gaps[r] = float(top2[1] - top2[0])
        weights = np.exp(values - values.max())
        scores[r] = weights[tok] / weights.sum()
        tokens.append(tok)
    return scores, tokens, gaps
