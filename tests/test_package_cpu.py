"""The execution-package reader on the host: a package written by the reference's own weight-store
writer and GraphIR emitter (tests/golden/make_package.py) yields the right geometry and bit-exact
tensors, and every tampered byte, size, digest or header is refused before loading."""
from __future__ import annotations

import json
import shutil

import numpy as np
import pytest

from diffusorrt_b200.package import read_package
from oracle.numerics import bf16_bits, synth_weights


@pytest.fixture(scope="module")
def pkg_dir(golden_dir):
    return golden_dir / "tiny_package"


def test_geometry_and_tensors(pkg_dir):
    from make_package import GEOMETRY, SEED, STD

    pkg = read_package(pkg_dir)
    for key, value in GEOMETRY.items():
        assert pkg.config[key] == value, key
    assert pkg.config["attention_mask_kind"] == "d2f_hybrid" and pkg.config["logits_shift"] is False
    want = synth_weights(GEOMETRY, SEED, **STD)
    assert set(pkg.tensors) == set(want)
    for name, arr in pkg.items():
        assert arr.dtype == np.uint16, name
        np.testing.assert_array_equal(arr, bf16_bits(want[name]).reshape(arr.shape))


def _copy(src, dst):
    shutil.copytree(src, dst)
    return dst


def test_tampered_shard_is_refused(pkg_dir, tmp_path):
    d = _copy(pkg_dir, tmp_path / "p")
    shard = sorted((d / "weights").glob("*.safetensors"))[1]
    raw = bytearray(shard.read_bytes())
    raw[-5] ^= 0x40
    shard.write_bytes(bytes(raw))
    with pytest.raises(ValueError, match="sha256"):
        read_package(d)


def test_truncated_shard_is_refused(pkg_dir, tmp_path):
    d = _copy(pkg_dir, tmp_path / "p")
    shard = sorted((d / "weights").glob("*.safetensors"))[0]
    shard.write_bytes(shard.read_bytes()[:-2])
    with pytest.raises(ValueError, match="size"):
        read_package(d)


def test_edited_index_is_refused(pkg_dir, tmp_path):
    d = _copy(pkg_dir, tmp_path / "p")
    index = d / "weights" / "weights.index.json"
    doc = json.loads(index.read_text())
    doc["shards"][0]["tensors"][0]["shape"] = [128, 256]
    index.write_text(json.dumps(doc, sort_keys=True, separators=(",", ":")) + "\n")
    with pytest.raises(ValueError, match="digest"):
        read_package(d)
    # with the manifest digest updated too, the shard header still disagrees
    import hashlib

    manifest = json.loads((d / "model.json").read_text())
    manifest["output_hash"] = hashlib.sha256(index.read_bytes()).hexdigest()
    (d / "model.json").write_text(json.dumps(manifest))
    with pytest.raises(ValueError, match="header"):
        read_package(d)


def test_reference_outside_the_package_is_refused(pkg_dir, tmp_path):
    d = _copy(pkg_dir, tmp_path / "p")
    manifest = json.loads((d / "model.json").read_text())
    manifest["merged_weights_ref"] = "../elsewhere/weights.index.json"
    (d / "model.json").write_text(json.dumps(manifest))
    with pytest.raises(ValueError, match="leaves"):
        read_package(d)
