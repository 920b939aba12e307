"""Execution-package reader: geometry and weights of a converted package, for ``Runtime(package_dir)``.

The SDK's converter writes (python/src/edllm/converter/convert_hf_masked_diffusion.py, the sharded
store of python/src/edllm/weight_store.py:35-40, 226-370, 393-530):

    model.json                  manifest: merged_weights_ref, output_hash (sha256 of the index),
                                package_format "safetensors_sharded_v1", weight_storage_dtype
                                "preserved", graph_ref
    graph.json                  the GraphIR: per-layer ops with their parameters and weight keys
    weights/weights.index.json  schema_version 1, format "safetensors", storage_dtype "preserved",
                                tensor_count, total_tensor_bytes, shards [{ref, sha256, byte_length,
                                tensors [{name, dtype, shape, byte_length}]}]
    weights/shard-NNNNN.safetensors

Every shard is verified against the index (size, sha256, and each tensor's dtype, shape and byte
length against the shard's own safetensors header) and the index against the manifest's digest
before any byte reaches the device; a mismatch raises ValueError. Files are opened relative to the
package directory and must stay inside it.

Geometry comes from the GraphIR and the tensor shapes: layer count, heads, head_dim, eps, RoPE theta,
QK-norm, q/k/v bias, the attention mask kind and the logits convention from graph.json; hidden size,
vocabulary and intermediate size from the embedding and gate_proj shapes; a tied lm_head when the
package's lm_head bytes equal the embedding's.
"""
from __future__ import annotations

import hashlib
import json
import mmap
import struct
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Iterator

import numpy as np

SHARDED_FORMAT = "safetensors_sharded_v1"
_DTYPES = {"bfloat16": ("BF16", np.uint16, 2), "float32": ("F32", np.float32, 4), "float16": ("F16", np.float16, 2)}


@dataclass
class TensorRecord:
    name: str
    dtype: str
    shape: tuple[int, ...]
    shard: Path
    offset: int          # byte offset of the data in the shard file
    nbytes: int


@dataclass
class Package:
    root: Path
    manifest: dict
    graph: dict
    tensors: dict[str, TensorRecord] = field(default_factory=dict)
    config: dict[str, Any] = field(default_factory=dict)

    def array(self, name: str) -> np.ndarray:
        """The tensor's stored values: uint16 bf16 bits for bfloat16, float32 / float16 otherwise."""
        rec = self.tensors[name]
        _, np_dtype, _ = _DTYPES[rec.dtype]
        with open(rec.shard, "rb") as f, mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) as mm:
            data = np.frombuffer(mm, dtype=np.uint8, count=rec.nbytes, offset=rec.offset).copy()
        return data.view(np_dtype).reshape(rec.shape)

    def items(self) -> Iterator[tuple[str, np.ndarray]]:
        for name in self.tensors:
            yield name, self.array(name)


def _inside(root: Path, ref: str) -> Path:
    path = (root / ref).resolve()
    if root.resolve() not in path.parents or path.is_symlink():
        raise ValueError(f"package reference {ref!r} leaves the package directory")
    return path


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 22), b""):
            h.update(chunk)
    return h.hexdigest()


def _shard_header(path: Path) -> tuple[dict, int]:
    """The safetensors header of a shard and the file offset where its data section starts."""
    with open(path, "rb") as f:
        head = f.read(8)
        if len(head) != 8:
            raise ValueError(f"{path.name}: truncated safetensors header")
        (n,) = struct.unpack("<Q", head)
        if n > 64 * 1024 * 1024:
            raise ValueError(f"{path.name}: safetensors header of {n} bytes")
        header = json.loads(f.read(n))
    return header, 8 + n


def _op_params(layer: dict, op_type: str, role: str | None = None) -> dict | None:
    for op in layer["ops"]:
        if op["type"] == op_type and (role is None or op["params"].get("role") == role):
            return op["params"]
    return None


def read_package(package_dir: str | Path) -> Package:
    root = Path(package_dir)
    manifest = json.loads((root / "model.json").read_text(encoding="utf-8"))
    if manifest.get("package_format") != SHARDED_FORMAT or manifest.get("weight_storage_dtype") != "preserved":
        raise ValueError("the package loader reads sharded safetensors packages (package_format "
                         f"{SHARDED_FORMAT!r}, weight_storage_dtype 'preserved')")
    index_path = _inside(root, manifest["merged_weights_ref"])
    digest = manifest.get("output_hash") or ""
    if digest and _sha256(index_path) != digest:
        raise ValueError("weight index digest does not match the manifest's output_hash")
    index = json.loads(index_path.read_text(encoding="utf-8"))
    if index.get("schema_version") != 1 or index.get("format") != "safetensors" or index.get("storage_dtype") != "preserved":
        raise ValueError("unsupported weight index (schema_version 1, safetensors, preserved dtypes)")
    graph = json.loads(_inside(root, manifest.get("graph_ref", "graph.json")).read_text(encoding="utf-8"))
    pkg = Package(root=root, manifest=manifest, graph=graph)
    total = 0
    for shard in index["shards"]:
        path = _inside(root, shard["ref"])
        if path.stat().st_size != shard["byte_length"]:
            raise ValueError(f"{shard['ref']}: size differs from the index")
        if _sha256(path) != shard["sha256"]:
            raise ValueError(f"{shard['ref']}: sha256 differs from the index")
        header, data0 = _shard_header(path)
        for t in shard["tensors"]:
            name, dtype = t["name"], t["dtype"]
            if dtype not in _DTYPES:
                raise ValueError(f"{name}: dtype {dtype} is not served")
            st_dtype, _, esize = _DTYPES[dtype]
            h = header.get(name)
            shape = tuple(int(d) for d in t["shape"])
            if h is None or h["dtype"] != st_dtype or tuple(h["shape"]) != shape:
                raise ValueError(f"{name}: the shard header disagrees with the index")
            lo, hi = (int(v) for v in h["data_offsets"])
            if hi - lo != t["byte_length"] or t["byte_length"] != esize * int(np.prod(shape, dtype=np.int64)):
                raise ValueError(f"{name}: byte length disagrees with its shape")
            if name in pkg.tensors:
                raise ValueError(f"{name}: stored twice")
            pkg.tensors[name] = TensorRecord(name, dtype, shape, path, data0 + lo, hi - lo)
            total += hi - lo
    if len(pkg.tensors) != index["tensor_count"] or total != index["total_tensor_bytes"]:
        raise ValueError("the shards do not hold the index's tensor set")
    pkg.config = _geometry(pkg)
    return pkg


def _geometry(pkg: Package) -> dict:
    g = pkg.graph
    layers = g["layers"]
    first = layers[0]
    attn = _op_params(first, "attention")
    gqa = _op_params(first, "gqa_repeat")
    rope = _op_params(first, "rope", "q")
    qk = _op_params(first, "qk_norm", "q")
    q_lin = _op_params(first, "linear", "q")
    embed_key = g["embedding"]["weight_keys"]["embedding"]
    lm_key = g["lm_head"]["weight_keys"]["weight"]
    V, H = pkg.tensors[embed_key].shape
    inter = pkg.tensors[f"model.layers.0.mlp.gate_proj.weight"].shape[0]
    tied = lm_key not in pkg.tensors or np.array_equal(pkg.array(lm_key), pkg.array(embed_key))
    convention = g.get("logits_convention", "raw")
    if convention not in ("raw", "dream_ar_shift"):
        raise ValueError(f"logits convention {convention!r} is not served")
    return dict(
        layer_count=len(layers), hidden_size=int(H), attention_heads=int(attn["n_heads"]),
        num_kv_heads=int(gqa["num_kv_heads"]) if gqa else int(attn["n_heads"]), head_dim=int(attn["head_dim"]),
        intermediate_size=int(inter), vocab_size=int(V), qk_norm=bool(qk and qk.get("apply_qk_norm")),
        qkv_bias=bool(q_lin and q_lin.get("bias_present")), tied_lm_head=bool(tied),
        rms_norm_eps=float(g["final_norm"]["params"].get("eps", 1e-6)),
        rope_theta=float(rope["rope_theta"]) if rope else 1e6,
        attention_mask_kind=attn.get("mask_kind", "d2f_hybrid"), logits_shift=convention == "dream_ar_shift",
    )
