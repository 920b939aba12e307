"""The C-ABI library builds, loads without a GPU and exports every symbol the header declares.
No compute calls are made here (there may be no GPU)."""
from __future__ import annotations

import ctypes
import json
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "diffusorrt_b200.h"


def _declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(drt_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from diffusorrt_b200 import _lib, build

    build.build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    names = _declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_the_header(lib):
    from diffusorrt_b200 import _lib

    assert sorted(_lib.SIGNATURES) == _declared_functions()


def test_abi_version_matches_reference(lib, golden_dir):
    meta = json.loads((golden_dir / "cases.json").read_text())
    a, b, c = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    assert lib.drt_abi_version(ctypes.byref(a), ctypes.byref(b), ctypes.byref(c)) == 0
    assert [a.value, b.value, c.value] == meta["abi_version"]


def test_status_and_enum_values_match_reference(golden_dir):
    meta = json.loads((golden_dir / "cases.json").read_text())
    text = HEADER.read_text()
    for name, value in meta["abi_status"].items():
        assert re.search(rf"DRT_{name}\s*=\s*{value}\b", text), name
    defines = dict(re.findall(r"#define (DRT_\w+) (\d+)", text))
    assert int(defines["DRT_STRATEGY_BLOCK_THRESHOLD"]) == meta["decode_strategy"]["block_threshold"]
    assert int(defines["DRT_STRATEGY_BD3_FIXED_QUOTA"]) == meta["decode_strategy"]["bd3_fixed_quota"]
    assert int(defines["DRT_STRATEGY_ENTROPY_COUNT"]) == meta["decode_strategy"]["entropy_count"]
    assert int(defines["DRT_COMMIT_THRESHOLD"]) == meta["commit_policy"]["threshold"]
    assert int(defines["DRT_COMMIT_FIXED_QUOTA"]) == meta["commit_policy"]["fixed_quota"]
    assert int(defines["DRT_MASK_BIDIRECTIONAL"]) == meta["attention_mask_kind"]["bidirectional"]
    assert int(defines["DRT_MASK_D2F_HYBRID"]) == meta["attention_mask_kind"]["d2f_hybrid"]


def test_struct_layouts_match_header(tmp_path):
    """The ctypes mirrors have the sizes and offsets the C compiler gives the header structs."""
    import shutil
    import subprocess

    from diffusorrt_b200 import _lib

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    structs = {"drt_model_config": _lib.ModelConfig, "drt_session_config": _lib.SessionConfig,
               "drt_generate_params": _lib.GenerateParams, "drt_generate_result": _lib.GenerateResult,
               "drt_step_trace": _lib.StepTrace, "drt_metrics": _lib.Metrics}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "diffusorrt_b200.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in py._fields_:
            lines.append(f'printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    for line in filter(None, out):
        cname, what, value = line.split()
        py = structs[cname]
        expect = ctypes.sizeof(py) if what == "size" else getattr(py, what).offset
        assert int(value) == expect, (cname, what)


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    from diffusorrt_b200 import _lib

    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setenv("DIFFUSORRT_B200_LIB", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.load()


@pytest.mark.parametrize("n_masked,steps,eps", [(256, 256, 1e-3), (256, 64, 1e-3), (64, 256, 1e-3), (7, 3, 0.5),
                                                (100, 100, 0.0), (33, 17, 1.0), (1, 1, 1e-3), (0, 5, 1e-3),
                                                (512, 300, 0.01)])
def test_entropy_count_schedule_matches_oracle(lib, n_masked, steps, eps):
    """The host schedule of the full-canvas loop (pure host code, no device call) equals the oracle's
    EntropyCount plan driven by a canvas that loses exactly the transfer count each step."""
    from oracle import policy as opol

    got = (ctypes.c_int32 * steps)()
    assert lib.drt_entropy_count_schedule(n_masked, steps, ctypes.c_double(eps), got) == 0
    mask = -1
    c = opol.Canvas([5] + [mask] * n_masked, 1, mask, -2)
    pol = opol.EntropyCount(eps=eps, steps=steps)
    want = []
    for step in range(steps):
        plan = pol.plan(c, step)
        if plan.action == "stop":
            want.append(0)
            continue
        if plan.action == "skip":
            want.append(0)
            continue
        k = min(pol._k, len(plan.frontier))
        want.append(k)
        for p in plan.frontier[:k]:
            c.x[p] = 1
    assert list(got) == want
    assert sum(want) == n_masked
