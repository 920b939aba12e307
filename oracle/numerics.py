"""bf16 rounding and the seeded synthetic weights, restated on the CPU (test infrastructure)."""
from __future__ import annotations

import math

import numpy as np

# Irwin-Hall sum of four uniform bytes has variance 4 * (256**2 - 1) / 12 = 21845.
UNIT_STD = math.sqrt(21845.0)
_K1 = np.uint64(0x9E3779B97F4A7C15)
_K2 = np.uint64(0xD1B54A32D192ED03)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)

# Tensor ids of the generator (must match drt_model_init_synthetic in csrc/capi.cu).
TID_EMBED = 1
TID_LM_HEAD = 2
LAYER_KINDS = ("q", "k", "v", "o", "gate", "up", "down", "bq", "bk", "bv")


def layer_tensor_id(layer: int, kind: str) -> int:
    return 16 + 16 * layer + LAYER_KINDS.index(kind)


def bf16_round(x) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even); result stays float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    bits = (bits + np.uint64(0x7FFF) + ((bits >> np.uint64(16)) & np.uint64(1))) & np.uint64(0xFFFF0000)
    out = bits.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out).astype(np.float32)


def bf16_bits(x) -> np.ndarray:
    """uint16 bf16 encodings of float32 values that are already bf16-representable."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    return (x.view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def from_bf16_bits(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def _mix64(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * _M1
    z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def synth_scale(std: float) -> np.float32:
    """The f32 multiplier of the generator: f32(f64(f32(std)) / sqrt(21845))."""
    return np.float32(float(np.float32(std)) / UNIT_STD)


def synth_tensor(seed: int, tensor_id: int, rows: int, cols: int, std: float, *, chunk: int = 1 << 24) -> np.ndarray:
    """[rows, cols] float32 array of bf16-representable synthetic weights."""
    n = rows * cols
    out = np.empty(n, dtype=np.float32)
    scale = synth_scale(std)
    base = None
    with np.errstate(over="ignore"):
        base = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) * _K1 + np.uint64(tensor_id) * _K2
        for lo in range(0, n, chunk):
            hi = min(n, lo + chunk)
            z = _mix64(base + np.arange(lo, hi, dtype=np.uint64))
            u = ((z & np.uint64(0xFF)) + ((z >> np.uint64(8)) & np.uint64(0xFF))
                 + ((z >> np.uint64(16)) & np.uint64(0xFF)) + ((z >> np.uint64(24)) & np.uint64(0xFF)))
            vals = (u.astype(np.int64) - 510).astype(np.float32) * scale
            out[lo:hi] = bf16_round(vals)
    return out.reshape(rows, cols)


def synth_weights(cfg: dict, seed: int, *, linear_std: float, embed_std: float, bias_std: float = 0.0) -> dict:
    """Weights dict keyed by package names, as drt_model_init_synthetic fills the device."""
    H = cfg["hidden_size"]
    nq, nkv, hd = cfg["attention_heads"], cfg["num_kv_heads"], cfg["head_dim"]
    inter = cfg["intermediate_size"]
    V = cfg["vocab_size"]
    w = {"model.embed_tokens.weight": synth_tensor(seed, TID_EMBED, V, H, embed_std)}
    if cfg.get("tied_lm_head", True):
        w["lm_head.weight"] = w["model.embed_tokens.weight"]
    else:
        w["lm_head.weight"] = synth_tensor(seed, TID_LM_HEAD, V, H, embed_std)
    w["model.norm.weight"] = np.ones(H, dtype=np.float32)
    for layer in range(cfg["layer_count"]):
        p = f"model.layers.{layer}."
        t = lambda kind: layer_tensor_id(layer, kind)  # noqa: E731
        w[p + "self_attn.q_proj.weight"] = synth_tensor(seed, t("q"), nq * hd, H, linear_std)
        w[p + "self_attn.k_proj.weight"] = synth_tensor(seed, t("k"), nkv * hd, H, linear_std)
        w[p + "self_attn.v_proj.weight"] = synth_tensor(seed, t("v"), nkv * hd, H, linear_std)
        w[p + "self_attn.o_proj.weight"] = synth_tensor(seed, t("o"), H, nq * hd, linear_std)
        w[p + "mlp.gate_proj.weight"] = synth_tensor(seed, t("gate"), inter, H, linear_std)
        w[p + "mlp.up_proj.weight"] = synth_tensor(seed, t("up"), inter, H, linear_std)
        w[p + "mlp.down_proj.weight"] = synth_tensor(seed, t("down"), H, inter, linear_std)
        w[p + "input_layernorm.weight"] = np.ones(H, dtype=np.float32)
        w[p + "post_attention_layernorm.weight"] = np.ones(H, dtype=np.float32)
        if cfg.get("qk_norm", False):
            w[p + "self_attn.q_norm.weight"] = np.ones(hd, dtype=np.float32)
            w[p + "self_attn.k_norm.weight"] = np.ones(hd, dtype=np.float32)
        if cfg.get("qkv_bias", False):
            w[p + "self_attn.q_proj.bias"] = synth_tensor(seed, t("bq"), 1, nq * hd, bias_std)[0]
            w[p + "self_attn.k_proj.bias"] = synth_tensor(seed, t("bk"), 1, nkv * hd, bias_std)[0]
            w[p + "self_attn.v_proj.bias"] = synth_tensor(seed, t("bv"), 1, nkv * hd, bias_std)[0]
    return w


def rope_half_tables(n_pos: int, head_dim: int, theta: float):
    """RoPE half tables [n_pos, head_dim/2] in the reference's float32 NumPy arithmetic
    (python/src/edllm/backends/mlx_forward.py:1566-1595, linear factor 1)."""
    half = head_dim // 2
    inv_freq = 1.0 / (theta ** (np.arange(0, half, dtype=np.float32) / half))
    inv_freq = inv_freq / max(1e-6, 1.0)
    freqs = np.einsum("i,j->ij", np.arange(n_pos, dtype=np.float32), inv_freq)
    return np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32)
