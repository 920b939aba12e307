"""Model geometries served by the engine and helpers shared by the runtime.

Geometry follows the reference runtime configs: Qwen3-0.6B BD3LM
(python/src/edllm/backends/cuda_profile.py:151-162, block 32, MASK 151669) and Dream-7B
(cuda_profile.py:63-74, MASK 151666). EOS 151645 is the `<|im_end|>` id of the Qwen3 case
fixtures; callers of a real tokenizer pass their own.
"""
from __future__ import annotations

import numpy as np

QWEN3_06B_BD3LM = dict(
    layer_count=28, hidden_size=1024, attention_heads=16, num_kv_heads=8, head_dim=128,
    intermediate_size=3072, vocab_size=151936, qk_norm=True, qkv_bias=False, tied_lm_head=True,
    rms_norm_eps=1e-6, rope_theta=1e6, mask_token_id=151669, eos_token_id=151645, block_size=32,
    logits_shift=False, mask_origin=0,
)

DREAM_7B = dict(
    layer_count=28, hidden_size=3584, attention_heads=28, num_kv_heads=4, head_dim=128,
    intermediate_size=18944, vocab_size=152064, qk_norm=False, qkv_bias=True, tied_lm_head=False,
    rms_norm_eps=1e-6, rope_theta=1e6, mask_token_id=151666, eos_token_id=151643, block_size=8,
    # Dream's logits convention (dream_ar_shift) and its D2F graph's mask origin (the prompt)
    logits_shift=True, mask_origin="prompt",
)

# Seeded synthetic weights: linears and embedding N(0, 0.02^2)-shaped (an Irwin-Hall sum of four
# bytes, scaled), norms 1, biases 0.02.
SYNTHETIC_STD = dict(linear_std=0.02, embed_std=0.02, bias_std=0.02)


def rope_half_tables(n_pos: int, head_dim: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    """cos / sin half tables [n_pos, head_dim / 2] computed in float32 exactly as the reference
    builds its RoPE tables (python/src/edllm/backends/mlx_forward.py:1566-1595, linear factor 1):
    inv_freq = 1 / theta ** (arange(half, f32) / half), angles = outer(arange(n_pos, f32), inv_freq)."""
    half = head_dim // 2
    inv_freq = 1.0 / (theta ** (np.arange(0, half, dtype=np.float32) / half))
    inv_freq = inv_freq / max(1e-6, 1.0)
    ang = np.einsum("i,j->ij", np.arange(n_pos, dtype=np.float32), inv_freq)
    return np.ascontiguousarray(np.cos(ang), dtype=np.float32), np.ascontiguousarray(np.sin(ang), dtype=np.float32)
