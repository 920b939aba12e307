"""Runtime(package_dir) on the GPU: a package in the reference's layout (tests/golden/tiny_package,
written by the reference's weight-store writer and GraphIR emitter) loads its geometry and verified
weights onto the device — the resident tensors equal the package's bytes — and its window forward
matches the oracle's forward of the same weights within the stated bf16 tolerance; the int8
weight-only precision quantizes the loaded weights."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from bf16_tolerance import assert_logits_close  # noqa: E402
from oracle import forward as ofwd  # noqa: E402
from oracle.numerics import from_bf16_bits  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pkg_dir(golden_dir):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import build

    build.build()
    return golden_dir / "tiny_package"


def _package_weights(pkg_dir):
    from diffusorrt_b200.package import read_package

    pkg = read_package(pkg_dir)
    return pkg.config, {name: from_bf16_bits(arr).astype(np.float32) for name, arr in pkg.items()}


def test_package_loads_onto_the_device(pkg_dir):
    from diffusorrt_b200 import Runtime

    cfg, w = _package_weights(pkg_dir)
    with Runtime(pkg_dir, max_seq=256, max_prefill_rows=128) as rt:
        assert rt.config["hidden_size"] == 128 and rt.config["tied_lm_head"]
        for name in ("model.embed_tokens.weight", "model.layers.0.self_attn.q_proj.weight",
                     "model.layers.0.mlp.up_proj.weight", "model.layers.0.mlp.down_proj.weight",
                     "model.layers.0.post_attention_layernorm.weight"):
            shape = w[name].shape if w[name].ndim == 2 else (1, w[name].shape[0])
            np.testing.assert_array_equal(rt.get_tensor(name, shape), w[name].reshape(shape))
        ids = [int(t) for t in np.random.default_rng(3).integers(0, 200, size=64)] + [250] * 32
        scope = list(range(64, 96))
        with rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
            res = s.execute_window(ids, scope, mask_geometry=(0, 32))
        got = np.frombuffer(res.logits, dtype="<f4").reshape(res.n_rows, res.n_vocab)
    full = dict(cfg, mask_token_id=250, eos_token_id=251)
    want = ofwd.forward_mlx(w, full, ids, prompt_len=0, block_size=32, output_rows=scope)
    assert_logits_close(got, want)


def test_package_with_int8_precision(pkg_dir):
    from diffusorrt_b200 import Runtime

    cfg, w = _package_weights(pkg_dir)
    precision = {"version": 1, "scheme": "int8_weight_only", "weight_type": "int8", "activation_type": "bf16",
                 "accumulation_type": "fp32"}
    with Runtime(pkg_dir, max_seq=256, max_prefill_rows=128, precision=precision,
                 engine_config={"compute_dtype": 0, "linear_quant_bits": 8, "linear_quant_group_size": 64}) as rt:
        assert rt.quantized and rt.quant_bits == 8
        ids = [int(t) for t in np.random.default_rng(4).integers(0, 200, size=96)]
        scope = [0, 31, 32, 95]
        with rt.session({"decode_strategy": "bd3_fixed_quota", "block_size": 32}) as s:
            res = s.execute_window(ids, scope, mask_geometry=(0, 32))
        got = np.frombuffer(res.logits, dtype="<f4").reshape(res.n_rows, res.n_vocab)
    want = ofwd.forward_mlx(w, cfg, ids, prompt_len=0, block_size=32, output_rows=scope,
                            quant=ofwd.quantized_weights(w, cfg, bits=8), quant_bits=8)
    assert_logits_close(got, want)
