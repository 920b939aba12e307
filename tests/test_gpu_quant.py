"""4-bit affine linear weights (the benchmark's quantized configuration) on the GPU through the C ABI:

* the device quantizer equals its NumPy restatement bit for bit (packed nibbles, bf16 scales
  and biases, including constant groups);
* the quantized decode linear equals y = x @ bf16(scale * q + bias)^T accumulated in f32 (its own
  operand rounding) tightly, and the reference's quantized-matmul contract (f32 activations,
  f32 dequantized weights) within the bf16 operand-rounding tolerance;
* a quantized model's window forward matches the CPU oracle's quantized forward within the stated
  bf16 tolerance, and its device decode is checked step by step along its trajectory.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import forward as ofwd  # noqa: E402
from oracle import policy as opol  # noqa: E402
from oracle import selector as osel  # noqa: E402
from oracle.numerics import bf16_round, synth_weights  # noqa: E402
from oracle.quant import dequantize, pack_q4, quantize_q4  # noqa: E402

from bf16_tolerance import assert_logits_close  # noqa: E402

pytestmark = pytest.mark.gpu

SMALL = dict(layer_count=2, hidden_size=256, attention_heads=4, num_kv_heads=2, head_dim=128,
             intermediate_size=512, vocab_size=4096, qk_norm=True, qkv_bias=False, tied_lm_head=True,
             rms_norm_eps=1e-6, rope_theta=1e6, mask_token_id=4000, eos_token_id=4001, block_size=32)
STD = dict(linear_std=0.05, embed_std=0.5)
SEED = 5


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import build
    build.build()
    return torch.device("cuda:0")


def _bf16(x: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(dev).to(torch.bfloat16)


def test_quantizer_matches_oracle_bit_for_bit(dev):
    from diffusorrt_b200 import kernels
    rng = np.random.default_rng(1)
    w = bf16_round(rng.standard_normal((384, 1024)).astype(np.float32) * 0.03)
    w[3, 64:128] = np.float32(0.0078125)            # constant group: scale 0
    w[7, :64] = bf16_round(np.linspace(-2, 5, 64, dtype=np.float32))
    q, s, b = kernels.quantize_q4(_bf16(w, dev))
    want_q, want_s, want_b = quantize_q4(w)
    np.testing.assert_array_equal(q.cpu().numpy(), pack_q4(want_q))
    np.testing.assert_array_equal(s.float().cpu().numpy(), want_s)
    np.testing.assert_array_equal(b.float().cpu().numpy(), want_b)


@pytest.mark.parametrize("rows,n,K,splits", [(32, 1024, 1024, 4), (17, 1024, 3072, 16), (64, 4096, 1024, 2),
                                             (1, 256, 512, 1)])
def test_linear_q4_matches_references(dev, rows, n, K, splits):
    from diffusorrt_b200 import kernels
    rng = np.random.default_rng(rows * 7 + n)
    w = bf16_round(rng.standard_normal((n, K)).astype(np.float32) * 0.02)
    x = bf16_round(rng.standard_normal((rows, K)).astype(np.float32))
    q, s, b = kernels.quantize_q4(_bf16(w, dev))
    y = kernels.linear_q4(_bf16(x, dev), q, s, b, splits=splits).cpu().numpy()
    qq, ss, bb = quantize_q4(w)
    # the kernel's own operands: bf16 x times bf16(scale * q + bias), f32 accumulation
    w_op = bf16_round(np.repeat(ss, 64, 1) * qq.astype(np.float32) + np.repeat(bb, 64, 1))
    ref = (x.astype(np.float64) @ w_op.astype(np.float64).T)
    scale = float(np.abs(ref).max())
    assert np.abs(y - ref).max() <= 2e-5 * scale, (np.abs(y - ref).max(), scale)
    # the reference contract: f32 activations times f32 dequantized weights
    mlx = x.astype(np.float64) @ dequantize(qq, ss, bb).astype(np.float64).T
    assert np.abs(y - mlx).max() <= 1e-2 * scale


@pytest.fixture(scope="module")
def qrt(dev):
    from diffusorrt_b200 import Runtime
    r = Runtime(model_config=SMALL, max_seq=512, max_prefill_rows=256,
                engine_config={"linear_quant_bits": 4, "linear_quant_group_size": 64})
    r.init_synthetic(SEED, **STD)
    r.quantize(4, 64)
    yield r
    r.close()


@pytest.fixture(scope="module")
def qweights():
    w = synth_weights(SMALL, SEED, **STD)
    return w, ofwd.quantized_weights(w, SMALL)


def _prompt(n, seed, vocab=4000):
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, size=n)]


def test_quantized_window_forward_matches_oracle(qrt, qweights):
    w, qw = qweights
    ids = _prompt(130, 9)
    for p in (100, 101, 120, 129):
        ids[p] = SMALL["mask_token_id"]
    scope = [0, 63, 64, 100, 101, 120, 129]
    with qrt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
        res = s.execute_window(ids, scope, mask_geometry=(0, 32))
    got = np.frombuffer(res.logits, dtype="<f4").reshape(res.n_rows, res.n_vocab)
    want = ofwd.forward_mlx(w, SMALL, ids, prompt_len=0, block_size=32, output_rows=scope, quant=qw)
    assert_logits_close(got, want)


def test_quantized_decode_along_trajectory(qrt, qweights):
    """BD3 fixed-quota decode with k = 2 commits per step on the quantized model (the cfg3 policy
    shape), checked step by step along the device trajectory against the oracle's quantized forward
    (tests/decode_check.py)."""
    from decode_check import check_bd3_trajectory

    w, qw = qweights
    prompt = _prompt(64, 13)
    gen, steps, bs = 64, 32, 32
    with qrt.session({"decode_strategy": "bd3_fixed_quota", "block_size": bs}) as s:
        dev_out = s.generate(prompt, max_tokens=gen, steps=steps, block_size=bs, trace_steps=256)
    report = check_bd3_trajectory(dev_out, w, SMALL, prompt, gen=gen, steps=steps, block_size=bs, quant=qw, quant_bits=4)
    assert report["steps"] == steps, report
