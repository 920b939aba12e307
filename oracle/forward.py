"""Transformer forward restated on the CPU (test infrastructure and the timed CPU baseline).

Two precision contracts:

* ``forward_mlx`` — the reference MLX path with bf16 resident weights
  (``python/src/edllm/backends/mlx_ops.py``, ``mlx_forward.py``): f32 embedding rows and residual
  stream; RMSNorm in f32 with the weight multiplied after the normalize (mlx_ops.py:21-35);
  every linear casts its f32 input to bf16, multiplies bf16 x bf16 with an f32 accumulator and
  returns the bf16-rounded result widened to f32, bias added in f32 (mlx_ops.py:97-130);
  per-head QK-RMSNorm then split-half RoPE in f32 with float32 angle tables
  (mlx_forward.py:1164-1361, 1566-1595); SDPA in f32 with the additive d2f_hybrid mask
  (mlx_ops.py:191-288, 347-443); SwiGLU in f32 (mlx_ops.py:147-154); f32 logits.
* ``forward_fp64`` — the float64 executable spec (``python/src/edllm/graph/numpyref.py``:
  op_rms_norm :80-85, op_rope_split_half :123-142 with float64 tables, attention :152-233,
  op_linear :236-241, op_mlp_swiglu :244-252, interpret_graph :507-559).
"""
from __future__ import annotations

import math

import numpy as np

from .numerics import bf16_round, rope_half_tables
from .quant import dequantize, dequantize_q8, quantize_q4, quantize_q8


def visible_mask(q_pos: np.ndarray, kv_len: int, *, prompt_len: int, block_size: int, bidirectional: bool) -> np.ndarray:
    """[len(q_pos), kv_len] bool: eff(p) = -1 if p < prompt_len else (p - prompt_len) // block;
    visible iff eff(key) <= eff(query); everything visible when bidirectional."""
    keys = np.arange(kv_len, dtype=np.int64)
    if bidirectional:
        return np.ones((len(q_pos), kv_len), dtype=bool)

    def eff(p):
        p = np.asarray(p, dtype=np.int64)
        return np.where(p < prompt_len, np.int64(-1), (p - prompt_len) // block_size)

    return eff(keys)[None, :] <= eff(q_pos)[:, None]


def _rms32(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    scale = np.float32(1.0) / np.sqrt(var + np.float32(eps))
    return (x * scale).astype(np.float32) * np.asarray(w, dtype=np.float32)


def _lin32(x: np.ndarray, w: np.ndarray, b=None) -> np.ndarray:
    y = bf16_round(bf16_round(x) @ np.asarray(w, dtype=np.float32).T)
    if b is not None:
        y = (y + np.asarray(b, dtype=np.float32)).astype(np.float32)
    return y


def _lin32q(x: np.ndarray, wq, b=None) -> np.ndarray:
    """Quantized linear (mx.quantized_matmul, mlx_ops.py:108-117): f32 activations times the f32
    dequantized weights, f32 result with no bf16 rounding, bias added in f32."""
    y = (np.asarray(x, dtype=np.float32) @ wq.T).astype(np.float32)
    if b is not None:
        y = (y + np.asarray(b, dtype=np.float32)).astype(np.float32)
    return y


def quantized_weights(weights: dict, cfg: dict, bits: int = 4) -> dict:
    """The dequantized f32 copies of every quantized linear (layer q/k/v/o, gate/up, down and
    lm_head; reference keys mlx_dream.py:2033-2087), keyed like ``weights``; ``bits`` 4 (4-bit affine)
    or 8 (int8 weight-only, bf16-exact values)."""
    out = {}
    keys = [k for k in weights if k.startswith("model.layers.") and k.endswith(
        (".q_proj.weight", ".k_proj.weight", ".v_proj.weight", ".o_proj.weight", ".gate_proj.weight",
         ".up_proj.weight", ".down_proj.weight"))]
    lm = weights.get("lm_head.weight", weights["model.embed_tokens.weight"])
    quant, deq = (quantize_q8, dequantize_q8) if bits == 8 else (quantize_q4, dequantize)
    for k in keys:
        out[k] = deq(*quant(weights[k]))
    out["lm_head.weight"] = deq(*quant(lm))
    return out


def _rope32(x: np.ndarray, cos_h: np.ndarray, sin_h: np.ndarray) -> np.ndarray:
    # x [S, heads, d]; cos_h/sin_h [S, d/2] -> full tables [S, 1, d]
    cos = np.concatenate([cos_h, cos_h], axis=-1)[:, None, :]
    sin = np.concatenate([sin_h, sin_h], axis=-1)[:, None, :]
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return (x * cos + rot * sin).astype(np.float32)


def _sdpa32(q, k, v, visible):
    # q [S, nq, d], k/v [T, nkv, d] -> [S, nq*d]
    S, nq, d = q.shape
    rep = nq // k.shape[1]
    kk = np.repeat(k, rep, axis=1)
    vv = np.repeat(v, rep, axis=1)
    scale = np.float32(1.0 / math.sqrt(d))
    scores = np.einsum("shd,thd->hst", q, kk, optimize=True).astype(np.float32) * scale
    scores = np.where(visible[None, :, :], scores, np.float32(-np.inf))
    scores = scores - scores.max(axis=-1, keepdims=True)
    e = np.exp(scores)
    p = e / e.sum(axis=-1, keepdims=True)
    out = np.einsum("hst,thd->shd", p, vv, optimize=True).astype(np.float32)
    return out.reshape(S, nq * d)


def _sdpa_bf16_operands(q, k, v, visible):
    """``_sdpa32`` with the operand roundings of a bf16 tensor-core attention: Q and K (after QK-norm
    and RoPE) rounded to bf16, scores accumulated in f32, the unnormalised softmax weights
    P = 2^(s * log2(e) / sqrt(d) - max) rounded to bf16, O = (P @ V) / sum(P) in f32. V rows are
    bf16-rounded linear outputs already. Everything else is the f32 contract."""
    S, nq, d = q.shape
    rep = nq // k.shape[1]
    qb, kb = bf16_round(q), bf16_round(k)
    kk = np.repeat(kb, rep, axis=1)
    vv = np.repeat(v, rep, axis=1)
    c = np.float32(math.log2(math.e) / math.sqrt(d))
    scores = np.einsum("shd,thd->hst", qb, kk, optimize=True).astype(np.float32)
    scores = np.where(visible[None, :, :], scores, np.float32(-np.inf))
    m = scores.max(axis=-1, keepdims=True) * c
    p = bf16_round(np.exp2((scores * c - m).astype(np.float32)))
    l = p.sum(axis=-1, keepdims=True, dtype=np.float32)
    out = np.einsum("hst,thd->hsd", p, vv, optimize=True).astype(np.float32) / l
    return np.transpose(out, (1, 0, 2)).reshape(S, nq * d).astype(np.float32)


ATTENTION_OPERANDS = {"f32": _sdpa32, "bf16": _sdpa_bf16_operands}


def forward_mlx(weights: dict, cfg: dict, token_ids, *, prompt_len: int = 0, block_size: int = 32,
                bidirectional: bool = False, output_rows=None, rope=None, quant: dict | None = None,
                attn_operands: str = "f32", quant_bits: int = 4) -> np.ndarray:
    """Logits [len(output_rows) (or S), V] f32 of a full-window forward (no cache). With ``quant``
    (``quantized_weights``), every quantized linear follows the quantized-matmul contract.
    ``attn_operands="bf16"`` rounds the attention's Q, K and softmax weights to bf16 as tensor-core
    operands (``_sdpa_bf16_operands``); the default is the reference's f32 attention."""
    sdpa = ATTENTION_OPERANDS[attn_operands]
    ids = np.asarray(token_ids, dtype=np.int64)
    S = len(ids)
    H, nq, nkv, d = cfg["hidden_size"], cfg["attention_heads"], cfg["num_kv_heads"], cfg["head_dim"]
    eps = float(cfg.get("rms_norm_eps", 1e-6))
    if rope is None:
        rope = rope_half_tables(S, d, float(cfg.get("rope_theta", 1e6)))
    cos_h, sin_h = rope[0][:S], rope[1][:S]
    vis = visible_mask(np.arange(S), S, prompt_len=prompt_len, block_size=block_size, bidirectional=bidirectional)
    h = np.asarray(weights["model.embed_tokens.weight"], dtype=np.float32)[ids].copy()
    for layer in range(cfg["layer_count"]):
        p = f"model.layers.{layer}."
        g = lambda key: weights.get(p + key)  # noqa: E731

        def lin(x, key, bias_key=None):
            b = g(bias_key) if bias_key else None
            if quant is not None:
                # 4-bit: the quantized-matmul contract; int8 weight-only: the bf16 linear contract
                # over the dequantized (bf16-exact) weights
                return _lin32q(x, quant[p + key], b) if quant_bits == 4 else _lin32(x, quant[p + key], b)
            return _lin32(x, g(key), b)

        n = _rms32(h, g("input_layernorm.weight"), eps)
        q = lin(n, "self_attn.q_proj.weight", "self_attn.q_proj.bias").reshape(S, nq, d)
        k = lin(n, "self_attn.k_proj.weight", "self_attn.k_proj.bias").reshape(S, nkv, d)
        v = lin(n, "self_attn.v_proj.weight", "self_attn.v_proj.bias").reshape(S, nkv, d)
        if g("self_attn.q_norm.weight") is not None:
            q = _rms32(q, g("self_attn.q_norm.weight"), eps)
            k = _rms32(k, g("self_attn.k_norm.weight"), eps)
        q = _rope32(q, cos_h, sin_h)
        k = _rope32(k, cos_h, sin_h)
        attn = sdpa(q, k, v, vis)
        h = (h + lin(attn, "self_attn.o_proj.weight")).astype(np.float32)
        n2 = _rms32(h, g("post_attention_layernorm.weight"), eps)
        gate = lin(n2, "mlp.gate_proj.weight")
        up = lin(n2, "mlp.up_proj.weight")
        act = (gate * (np.float32(1.0) / (np.float32(1.0) + np.exp(-gate))) * up).astype(np.float32)
        h = (h + lin(act, "mlp.down_proj.weight")).astype(np.float32)
    rows = np.arange(S) if output_rows is None else np.asarray(output_rows, dtype=np.int64)
    hn = _rms32(h[rows], weights["model.norm.weight"], eps)
    if quant is not None:
        return _lin32q(hn, quant["lm_head.weight"]) if quant_bits == 4 else _lin32(hn, quant["lm_head.weight"])
    return _lin32(hn, weights["lm_head.weight"])


def forward_fp64(weights: dict, cfg: dict, token_ids, *, prompt_len: int = 0, block_size: int = 32,
                 bidirectional: bool = False, output_rows=None, cast=None) -> np.ndarray:
    """Float64 logits of the executable spec. ``cast(key)`` may supply cached float64 weights."""
    ids = np.asarray(token_ids, dtype=np.int64)
    S = len(ids)
    H, nq, nkv, d = cfg["hidden_size"], cfg["attention_heads"], cfg["num_kv_heads"], cfg["head_dim"]
    eps = float(cfg.get("rms_norm_eps", 1e-6))
    theta = float(cfg.get("rope_theta", 1e6))
    W = cast or (lambda key: None if weights.get(key) is None else np.asarray(weights[key], dtype=np.float64))

    def rms(x, w):
        var = np.mean(x * x, axis=-1, keepdims=True)
        return x / np.sqrt(var + eps) * w

    half = d // 2
    inv = 1.0 / (theta ** (np.arange(0, half, dtype=np.float64) / half))
    ang = np.einsum("i,j->ij", np.arange(S, dtype=np.float64), inv)
    cos, sin = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]

    def rope(x):
        out = np.empty_like(x)
        out[..., :half] = x[..., :half] * cos - x[..., half:] * sin
        out[..., half:] = x[..., :half] * sin + x[..., half:] * cos
        return out

    vis = visible_mask(np.arange(S), S, prompt_len=prompt_len, block_size=block_size, bidirectional=bidirectional)
    bias = np.where(vis, 0.0, -np.inf)
    h = W("model.embed_tokens.weight")[ids]
    for layer in range(cfg["layer_count"]):
        p = f"model.layers.{layer}."

        def lin(x, key, bkey=None):
            y = x @ W(p + key).T
            b = W(p + bkey) if bkey else None
            return y if b is None else y + b

        n = rms(h, W(p + "input_layernorm.weight"))
        q = lin(n, "self_attn.q_proj.weight", "self_attn.q_proj.bias").reshape(S, nq, d)
        k = lin(n, "self_attn.k_proj.weight", "self_attn.k_proj.bias").reshape(S, nkv, d)
        v = lin(n, "self_attn.v_proj.weight", "self_attn.v_proj.bias").reshape(S, nkv, d)
        if W(p + "self_attn.q_norm.weight") is not None:
            q = rms(q, W(p + "self_attn.q_norm.weight"))
            k = rms(k, W(p + "self_attn.k_norm.weight"))
        q, k = rope(q), rope(k)
        rep = nq // nkv
        kk, vv = np.repeat(k, rep, axis=1), np.repeat(v, rep, axis=1)
        sc = np.einsum("thd,shd->hts", q, kk, optimize=True) / math.sqrt(float(d)) + bias
        sc = np.exp(sc - sc.max(axis=-1, keepdims=True))
        pr = sc / sc.sum(axis=-1, keepdims=True)
        attn = np.einsum("hts,shd->thd", pr, vv, optimize=True).reshape(S, nq * d)
        h = h + attn @ W(p + "self_attn.o_proj.weight").T
        n2 = rms(h, W(p + "post_attention_layernorm.weight"))
        gate = n2 @ W(p + "mlp.gate_proj.weight").T
        up = n2 @ W(p + "mlp.up_proj.weight").T
        h = h + (gate / (1.0 + np.exp(-gate)) * up) @ W(p + "mlp.down_proj.weight").T
    rows = np.arange(S) if output_rows is None else np.asarray(output_rows, dtype=np.int64)
    hn = rms(h[rows], W("model.norm.weight"))
    return hn @ W("lm_head.weight").T


def dream_raw_rows(positions) -> list[int]:
    """Raw logits row each position reads under dream_ar_shift (shift_logits_for_dream,
    python/src/edllm/backends/mlx_ops.py:157-159: concatenate(logits[:1], logits[:-1])):
    position p reads raw row max(p - 1, 0)."""
    return [max(int(p) - 1, 0) for p in positions]


class PrefixKV:
    """K (after QK-norm and RoPE) and V of canvas positions [0, length) for every layer, float32:
    the exact prefix K/V of the reference's d2f path (PrefixKVCacheStrategy,
    python/src/edllm/backends/mlx_state_cache.py:51-515; the exact-D2F pattern of
    mlx_d2f_forward.py:205-368). Rows enter only once their tokens are final."""

    def __init__(self, cfg: dict):
        self.k = [None] * cfg["layer_count"]
        self.v = [None] * cfg["layer_count"]
        self.length = 0


def forward_mlx_cached(weights: dict, cfg: dict, token_ids, cache: PrefixKV, *, frozen: int, output_rows,
                       prompt_len: int = 0, block_size: int = 32, rope=None, attn_operands: str = "f32",
                       quant: dict | None = None, quant_bits: int = 4) -> np.ndarray:
    """``forward_mlx`` logits of ``output_rows`` (absolute positions) for the window ``token_ids``,
    computing only rows [cache.length, len(token_ids)) against the cached K/V, then caching the
    rows [cache.length, frozen) (final tokens). Under the block-causal d2f mask a cached row never
    attends past the frozen prefix, so this equals the cache-free forward (up to float32 summation
    order)."""
    ids = np.asarray(token_ids, dtype=np.int64)
    n = len(ids)
    c0 = cache.length
    if not c0 <= frozen <= n:
        raise ValueError("frozen prefix outside [cache length, window]")
    H, nq, nkv, d = cfg["hidden_size"], cfg["attention_heads"], cfg["num_kv_heads"], cfg["head_dim"]
    eps = float(cfg.get("rms_norm_eps", 1e-6))
    if rope is None:
        rope = rope_half_tables(n, d, float(cfg.get("rope_theta", 1e6)))
    cos_h, sin_h = rope[0][c0:n], rope[1][c0:n]
    S = n - c0
    vis = visible_mask(np.arange(c0, n), n, prompt_len=prompt_len, block_size=block_size, bidirectional=False)
    h = np.asarray(weights["model.embed_tokens.weight"], dtype=np.float32)[ids[c0:]].copy()
    for layer in range(cfg["layer_count"]):
        p = f"model.layers.{layer}."
        g = lambda key: weights.get(p + key)  # noqa: E731

        def lin(x, key, bias_key=None):
            b = g(bias_key) if bias_key else None
            if quant is not None:
                return _lin32q(x, quant[p + key], b) if quant_bits == 4 else _lin32(x, quant[p + key], b)
            return _lin32(x, g(key), b)

        x1 = _rms32(h, g("input_layernorm.weight"), eps)
        q = lin(x1, "self_attn.q_proj.weight", "self_attn.q_proj.bias").reshape(S, nq, d)
        k = lin(x1, "self_attn.k_proj.weight", "self_attn.k_proj.bias").reshape(S, nkv, d)
        v = lin(x1, "self_attn.v_proj.weight", "self_attn.v_proj.bias").reshape(S, nkv, d)
        if g("self_attn.q_norm.weight") is not None:
            q = _rms32(q, g("self_attn.q_norm.weight"), eps)
            k = _rms32(k, g("self_attn.k_norm.weight"), eps)
        q = _rope32(q, cos_h, sin_h)
        k = _rope32(k, cos_h, sin_h)
        k_all = k if cache.k[layer] is None else np.concatenate([cache.k[layer], k], axis=0)
        v_all = v if cache.v[layer] is None else np.concatenate([cache.v[layer], v], axis=0)
        attn = ATTENTION_OPERANDS[attn_operands](q, k_all, v_all, vis)
        h = (h + lin(attn, "self_attn.o_proj.weight")).astype(np.float32)
        x2 = _rms32(h, g("post_attention_layernorm.weight"), eps)
        gate = lin(x2, "mlp.gate_proj.weight")
        up = lin(x2, "mlp.up_proj.weight")
        act = (gate * (np.float32(1.0) / (np.float32(1.0) + np.exp(-gate))) * up).astype(np.float32)
        h = (h + lin(act, "mlp.down_proj.weight")).astype(np.float32)
        if frozen > c0:
            cache.k[layer] = k_all[:frozen]
            cache.v[layer] = v_all[:frozen]
    cache.length = max(c0, frozen)
    rows = np.asarray(output_rows, dtype=np.int64) - c0
    if rows.min(initial=0) < 0:
        raise ValueError("output rows inside the cached prefix")
    hn = _rms32(h[rows], weights["model.norm.weight"], eps)
    if quant is not None:
        return _lin32q(hn, quant["lm_head.weight"]) if quant_bits == 4 else _lin32(hn, quant["lm_head.weight"])
    return _lin32(hn, weights["lm_head.weight"])
