"""Deterministic stand-in forward for decode-loop golden traces (test infrastructure).

Logits for a window depend only on the token ids handed in (a CRC of their bytes seeds a
NumPy generator), so the reference loop and the restated loop see identical logits whenever
they reach identical canvases.
"""
from __future__ import annotations

import zlib

import numpy as np


def fake_logits(ids, vocab: int, *, scale: float = 3.0, bias_token: int | None = None, bias: float = 0.0) -> np.ndarray:
    arr = np.asarray(ids, dtype=np.int64)
    seed = zlib.crc32(arr.tobytes()) ^ (vocab * 2654435761 & 0xFFFFFFFF)
    rng = np.random.default_rng(seed)
    out = rng.normal(0.0, scale, size=(len(arr), vocab)).astype(np.float32)
    if bias_token is not None:
        out[:, bias_token] += np.float32(bias)
    return out
