"""Error model of the device's split entropy confidence (csrc/selector.cuh, sel_pass1_kernel<false,
true> + sel_entropy_kernel), restated in NumPy with the kernel's float32 steps, against the
reference's per-logit float64 sum (python/src/edllm/backends/diffusion_runtime.py:90-114):

    H = sum p log(p + eps) = [sum e (a - m)] / S - log S  +  sum p log1p(eps / p)

The first part is float64 from pass 1's chunk statistics. The second is at most V eps; the kernel
evaluates each of its terms divided by eps in float32 (d = log2(p / eps), q = 2^-|d|, log1p(q) as
2 atanh(q / (2 + q)) through s^14 / 15) and sums them in float64. The check: the split H lies
within 1e-3 of a float32 ulp of the reference's float64 H, for logit spreads from flat to peaked
and for T = 1 and T = 0.2, so the float32 cast both sides take agrees except within that margin of a
rounding boundary.
"""
from __future__ import annotations

import numpy as np
import pytest

f32 = np.float32
EPS = 1e-10
CHUNK = 8192


def _split_entropy(x32: np.ndarray, inv_t: float) -> float:
    x = x32.astype(np.float64) * inv_t
    stats = []
    for lo in range(0, x.size, CHUNK):  # pass 1: chunk max, sum e, sum e z (z clamped at -708)
        xc = x[lo:lo + CHUNK]
        mc = xc.max()
        z = np.maximum(xc - mc, -708.0)
        e = np.exp(z)
        stats.append((mc, e.sum(), (e * z).sum()))
    gm = max(m for m, _, _ in stats)
    S = T = 0.0
    for mc, sc, ac in stats:
        f = np.exp(mc - gm)
        S += sc * f
        T += f * (ac + (mc - gm) * sc)
    exact = T / S - np.log(S)
    # pass 2, float32 per logit
    s1 = inv_t * 1.4426950408889634
    s1h = f32(s1)
    s1l = f32(s1 - np.float64(s1h))
    c0 = -(np.log2(S) + np.log2(EPS))
    c0h = f32(c0)
    c0l = f32(c0 - np.float64(c0h))
    dx = (x32 - f32(x32.max())).astype(f32)
    with np.errstate(invalid="ignore"):
        d = (dx * s1h + c0h).astype(f32) + (dx * s1l + c0l).astype(f32)
    with np.errstate(invalid="ignore"):  # -inf x (s1h + s1l) of an excluded column: NaN, which fmaxf caps
        w = np.fmax(-np.abs(d), f32(-200)).astype(f32)
    q = np.where(w < -126, f32(0), np.exp2(w)).astype(f32)
    r = (f32(1) / (f32(2) + q)).astype(f32)
    s = (q * r).astype(f32)
    t = (s * s).astype(f32)
    P = np.full_like(t, f32(1 / 15))
    for c in (1 / 13, 1 / 11, 1 / 9, 1 / 7, 1 / 5, 1 / 3, 1.0):
        P = (P * t + f32(c)).astype(f32)
    g = np.where(d >= 0, f32(2) * r * P, q * ((f32(2) * s) * P + (-w) * f32(0.6931471805599453))).astype(f32)
    return exact + float(g.astype(np.float64).sum()) * EPS


@pytest.mark.parametrize("sd,temperature", [(3.0, 1.0), (1.0, 1.0), (10.0, 1.0), (0.3, 1.0), (1.0, 0.2), (3.0, 0.2)])
def test_split_entropy_within_float32_margin(sd, temperature):
    rng = np.random.default_rng(int(sd * 10) + int(temperature * 100))
    x = (rng.standard_normal(151936, dtype=np.float32) * f32(sd)).astype(f32)
    x[17] = -np.inf  # an excluded column scores p = 0
    inv_t = 1.0 / temperature
    a = x.astype(np.float64) * inv_t
    with np.errstate(invalid="ignore"):
        p = np.exp(a - a.max())
    p /= p.sum()
    ref = float(np.sum(p * np.log(p + 1e-10)))
    got = _split_entropy(x, inv_t)
    ulp = float(np.spacing(f32(abs(ref))))
    assert abs(got - ref) <= 1e-3 * ulp, (got, ref, abs(got - ref) / ulp)
