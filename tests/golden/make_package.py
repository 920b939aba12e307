"""Write a tiny execution package in the reference's on-disk layout, for the package-loader tests.

The weights go through the reference's own writer (``write_safetensors_weight_store``,
python/src/edllm/weight_store.py:393-530: ``weights/weights.index.json`` plus safetensors shards,
bf16 preserved, tied embedding declared), the graph through its GraphIR emitter
(python/src/edllm/graph/emitter.py ``build_graph_ir``), and model.json carries the manifest fields the
reference's converter records for a sharded store (python/src/edllm/converter/convert_hf_masked_diffusion.py:
merged_weights_ref, output_hash, package_format, weight_storage_dtype, graph_ref, model_config). The
values are the seeded synthetic weights of oracle/numerics.py (seed 9, linear std 0.05, embedding std
0.5), small enough to commit (a one-layer, hidden-128 model; shards of at most 160 KB so that there
are several). The reference tree is only read; nothing here runs on the GPU box.

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_package.py --reference /path/to/reference
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

OUT = HERE / "tiny_package"
GEOMETRY = dict(layer_count=1, hidden_size=128, attention_heads=1, num_kv_heads=1, head_dim=128, intermediate_size=128,
                vocab_size=256, rms_norm_eps=1e-6, rope_theta=1e6, qk_norm=True, qkv_bias=False, tied_lm_head=True)
SEED, STD = 9, dict(linear_std=0.05, embed_std=0.5)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DIFFUSORRT_REFERENCE"),
                    help="checkout of the reference project (or set DIFFUSORRT_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference checkout with --reference or DIFFUSORRT_REFERENCE")
    sys.path.insert(0, str(Path(args.reference) / "python" / "src"))
    sys.dont_write_bytecode = True
    import torch
    from edllm.graph.emitter import build_graph_ir
    from edllm.weight_store import write_safetensors_weight_store

    from oracle.numerics import synth_weights

    if OUT.exists():
        shutil.rmtree(OUT)
    OUT.mkdir()
    weights = synth_weights(GEOMETRY, SEED, **STD)
    graph = build_graph_ir(dict(GEOMETRY, uses_qk_norm=True, uses_shifted_logits=False, bias_present=False,
                                attention_mask_kind="d2f_hybrid"))

    def items():
        for name in sorted(weights):
            yield name, torch.from_numpy(np.ascontiguousarray(weights[name], dtype=np.float32)).to(torch.bfloat16)

    written = write_safetensors_weight_store(OUT, items(), tied_weight_keys=("model.embed_tokens.weight", "lm_head.weight"),
                                             max_shard_bytes=160 * 1024)
    manifest = {
        "version": {"major": 2, "minor": 0, "patch": 0},
        "decode_family": "masked_diffusion",
        "merged_weights_ref": written.spec.primary_ref,
        "output_hash": written.spec.digest,
        "package_format": written.spec.format,
        "weight_storage_dtype": written.spec.storage_dtype,
        "graph_ref": "graph.json",
        "ir_version": dict(graph.ir_version),
        "model_config": {"num_hidden_layers": 1, "hidden_size": 128, "num_attention_heads": 1, "num_key_value_heads": 1,
                         "head_dim": 128, "intermediate_size": 128, "vocab_size": 256, "rms_norm_eps": 1e-6,
                         "rope_theta": 1e6, "tie_word_embeddings": True},
        "synthetic_weights": {"seed": SEED, **STD},
    }
    (OUT / "model.json").write_text(json.dumps(manifest, indent=2), encoding="utf-8", newline="\n")
    (OUT / "graph.json").write_text(graph.to_json(indent=2), encoding="utf-8", newline="\n")
    print("package written to", OUT, "shards:", len(list((OUT / "weights").glob("*.safetensors"))))


if __name__ == "__main__":
    main()
