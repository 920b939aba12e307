"""The CUDA int8_weight_only precision (python/src/edllm/backends/device_runtime.py:19-56: int8 linear
weights with one absmax scale per group of 64 inputs, bf16 activations, f32 accumulation) on the GPU
through the C ABI:

* the device quantizer equals its NumPy restatement (oracle/quant.py quantize_q8) bit for bit,
  including constant and zero groups;
* the int8 decode linear equals y = bf16(x @ bf16(scale * (byte - 128))^T) with f32 accumulation;
* a Runtime opened with the SDK's precision descriptor and engine config for int8_weight_only runs
  window forwards within the stated bf16 tolerance of the oracle's int8 forward, and a whole BD3 decode
  checked step by step along the device trajectory.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from bf16_tolerance import assert_logits_close  # noqa: E402
from oracle import forward as ofwd  # noqa: E402
from oracle.numerics import bf16_round, synth_weights  # noqa: E402
from oracle.quant import dequantize_q8, quantize_q8  # noqa: E402

pytestmark = pytest.mark.gpu

SMALL = dict(layer_count=2, hidden_size=256, attention_heads=4, num_kv_heads=2, head_dim=128,
             intermediate_size=512, vocab_size=4096, qk_norm=True, qkv_bias=False, tied_lm_head=True,
             rms_norm_eps=1e-6, rope_theta=1e6, mask_token_id=4000, eos_token_id=4001, block_size=32)
STD = dict(linear_std=0.05, embed_std=0.5)
SEED = 6
# cuda_precision_descriptor("int8_weight_only") and cuda_engine_config (device_runtime.py:19-56)
PRECISION = {"version": 1, "scheme": "int8_weight_only", "weight_type": "int8", "activation_type": "bf16",
             "accumulation_type": "fp32", "scale_granularity": "per_group",
             "scale_layout": "row-major-linear-input-groups-g64", "calibration_provenance": "weight-group-absmax-v1"}
ENGINE = {"compute_dtype": 0, "d2f_exact_kv_cache": 0, "linear_quant_bits": 8, "linear_quant_group_size": 64}


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import build
    build.build()
    return torch.device("cuda:0")


def _bf16(x: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(dev).to(torch.bfloat16)


def test_q8_quantizer_matches_oracle_bit_for_bit(dev):
    from diffusorrt_b200 import kernels
    rng = np.random.default_rng(2)
    w = bf16_round(rng.standard_normal((256, 1024)).astype(np.float32) * 0.03)
    w[3, 64:128] = np.float32(0.0078125)   # constant group
    w[5, 128:192] = np.float32(0.0)        # zero group: scale 0
    w[7, :64] = bf16_round(np.linspace(-2, 5, 64, dtype=np.float32))
    q, s, b = kernels.quantize_q8(_bf16(w, dev))
    want_q, want_s, want_b = quantize_q8(w)
    np.testing.assert_array_equal(q.cpu().numpy(), want_q)
    np.testing.assert_array_equal(s.float().cpu().numpy(), want_s)
    np.testing.assert_array_equal(b.float().cpu().numpy(), want_b)
    # the dequantized values are within half a quantization step of the weights
    err = np.abs(dequantize_q8(want_q, want_s, want_b) - w)
    assert np.all(err <= np.repeat(want_s, 64, 1) * 0.5 + np.abs(w) * 2.0 ** -8)


@pytest.mark.parametrize("rows,n,K,splits", [(32, 1024, 1024, 4), (17, 1024, 3072, 16), (64, 4096, 1024, 2)])
def test_linear_q8_matches_its_contract(dev, rows, n, K, splits):
    from diffusorrt_b200 import kernels
    rng = np.random.default_rng(rows * 11 + n)
    w = bf16_round(rng.standard_normal((n, K)).astype(np.float32) * 0.02)
    x = bf16_round(rng.standard_normal((rows, K)).astype(np.float32))
    q, s, b = kernels.quantize_q8(_bf16(w, dev))
    y = kernels.linear_q8(_bf16(x, dev), q, s, b, splits=splits).cpu().numpy()
    w_op = dequantize_q8(*quantize_q8(w))
    ref = bf16_round((x.astype(np.float64) @ w_op.astype(np.float64).T).astype(np.float32))
    # f32 accumulation order against a float64 sum: the bf16 output differs by at most one ulp
    np.testing.assert_allclose(y, ref, rtol=2.0 ** -7, atol=1e-6)
    assert np.mean(y == ref) > 0.99


@pytest.fixture(scope="module")
def q8rt(dev):
    from diffusorrt_b200 import Runtime
    r = Runtime(model_config=SMALL, max_seq=512, max_prefill_rows=256, precision=PRECISION, engine_config=ENGINE,
                synthetic_seed=SEED)
    r.init_synthetic(SEED, **STD)
    assert r.quantized and r.quant_bits == 8
    yield r
    r.close()


@pytest.fixture(scope="module")
def q8weights():
    w = synth_weights(SMALL, SEED, **STD)
    return w, ofwd.quantized_weights(w, SMALL, bits=8)


def _prompt(n, seed, vocab=4000):
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, size=n)]


def test_q8_window_forward_matches_oracle(q8rt, q8weights):
    w, qw = q8weights
    ids = _prompt(130, 19)
    for p in (100, 101, 120, 129):
        ids[p] = SMALL["mask_token_id"]
    scope = [0, 63, 64, 100, 101, 120, 129]
    with q8rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
        res = s.execute_window(ids, scope, mask_geometry=(0, 32))
    got = np.frombuffer(res.logits, dtype="<f4").reshape(res.n_rows, res.n_vocab)
    want = ofwd.forward_mlx(w, SMALL, ids, prompt_len=0, block_size=32, output_rows=scope, quant=qw, quant_bits=8)
    assert_logits_close(got, want)


def test_q8_decode_along_trajectory(q8rt, q8weights):
    from decode_check import check_bd3_trajectory

    w, qw = q8weights
    prompt = _prompt(64, 23)
    with q8rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
        dev_out = s.generate(prompt, max_tokens=64, steps=32, block_size=32, trace_steps=64)
    report = check_bd3_trajectory(dev_out, w, SMALL, prompt, gen=64, steps=32, block_size=32, quant=qw, quant_bits=8)
    assert report["steps"] == 32, report
