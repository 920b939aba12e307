"""4-bit affine weight quantization restated in NumPy (test infrastructure).

The reference quantizes every layer linear and lm_head at load time
(``python/src/edllm/backends/mlx_dream.py:2090-2108`` via ``mlx_ops.quantize_linear_weight``,
``mlx_ops.py:63-94``) into per-group scale and bias in the weight dtype with
w ~ scale * q + bias, q in [0, 15]. The rounding rules live in ``mx.quantize`` (MLX, not in the
reference sources; parity of those rules is unpinned), so the build defines them from that affine
form and this module restates the build's definition operation by operation
(``diffusorrt_b200/csrc/quant.cuh``), in float32:

    lo, hi = min, max of the 64 bf16 weights of a group
    scale = bf16_round((hi - lo) / 15);  bias = bf16_round(lo)
    q = clip(rint((w - bias) / scale), 0, 15)        (q = 0 where scale == 0)
"""
from __future__ import annotations

import numpy as np

from .numerics import bf16_round

GROUP = 64


def quantize_q4(w) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """w [n, K] (bf16 values, any float dtype) -> q uint8 [n, K], scale / bias f32 [n, K // 64]
    holding bf16 values."""
    w = np.asarray(bf16_round(np.asarray(w, dtype=np.float32)), dtype=np.float32)
    n, K = w.shape
    if K % GROUP:
        raise ValueError("in-dim must be a multiple of 64")
    g = w.reshape(n, K // GROUP, GROUP)
    lo = g.min(axis=-1)
    hi = g.max(axis=-1)
    scale = bf16_round((hi - lo).astype(np.float32) / np.float32(15.0))
    bias = bf16_round(lo)
    with np.errstate(divide="ignore", invalid="ignore"):
        t = np.rint(((g - bias[..., None]).astype(np.float32) / scale[..., None]).astype(np.float32))
    t = np.where(scale[..., None] > 0, t, 0.0)
    q = np.clip(t, 0, 15).astype(np.uint8).reshape(n, K)
    return q, scale.astype(np.float32), bias.astype(np.float32)


def pack_q4(q: np.ndarray) -> np.ndarray:
    """uint8 [n, K] -> [n, K // 2]: input 2j in the low nibble of byte j."""
    return (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)


def dequantize(q: np.ndarray, scale: np.ndarray, bias: np.ndarray) -> np.ndarray:
    """float32 weights scale * q + bias (the quantized matmul's weight values)."""
    n, K = q.shape
    s = np.repeat(scale, GROUP, axis=1)
    b = np.repeat(bias, GROUP, axis=1)
    return (s * q.astype(np.float32)).astype(np.float32) + b


def quantize_q8(w) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """int8 weight-only quantization (the build's definition, ``quant.cuh``), in float32:
        amax = max |w| of the 64 bf16 weights of a group;  scale = bf16_round(amax / 127)
        q = clip(rint(w / scale), -127, 127)                  (q = 0 where scale == 0)
    returned as the stored bytes q + 128 (uint8 [n, K]), scale and bias = -128 * scale (f32 [n, K // 64]
    holding bf16 values)."""
    w = np.asarray(bf16_round(np.asarray(w, dtype=np.float32)), dtype=np.float32)
    n, K = w.shape
    if K % GROUP:
        raise ValueError("in-dim must be a multiple of 64")
    g = w.reshape(n, K // GROUP, GROUP)
    amax = np.abs(g).max(axis=-1)
    scale = bf16_round(amax.astype(np.float32) / np.float32(127.0))
    with np.errstate(divide="ignore", invalid="ignore"):
        t = np.rint((g / scale[..., None]).astype(np.float32))
    t = np.where(scale[..., None] > 0, t, 0.0)
    q = (np.clip(t, -127, 127) + 128).astype(np.uint8).reshape(n, K)
    return q, scale.astype(np.float32), (np.float32(-128.0) * scale).astype(np.float32)


def dequantize_q8(q: np.ndarray, scale: np.ndarray, bias: np.ndarray) -> np.ndarray:
    """The int8 weight-only linear's weight values: bf16_round(scale * byte + bias) = bf16_round(scale
    * (byte - 128)), the bf16 operand the tensor cores take."""
    s = np.repeat(scale, GROUP, axis=1)
    b = np.repeat(bias, GROUP, axis=1)
    return bf16_round((s * q.astype(np.float32)).astype(np.float32) + b)
