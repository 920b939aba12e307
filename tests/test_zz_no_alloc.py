"""The allocation-free selector entry point, drt_selector_rows_noalloc.

Some callers of this library may not allocate device memory: a host that owns all GPU memory
through its own pool or a fixed budget, or a latency-critical caller that cannot accept
cudaMalloc's implicit synchronization. For them the selector keeps its scratch in a static device
array. These tests call it through the C ABI and check it against drt_selector_rows (caller
scratch) on two calls in a row, so the second call also shows that the reused array was reset.
This file is collected last on purpose.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import _lib, build

    build.build()
    return _lib.load()


def _with_scratch(lib, x, mode, temperature):
    rows, vocab = x.shape
    scratch = torch.empty(int(lib.drt_selector_scratch_bytes(rows, vocab)), dtype=torch.uint8, device=x.device)
    conf = torch.empty(rows, dtype=torch.float64, device=x.device)
    tok = torch.empty(rows, dtype=torch.int32, device=x.device)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.drt_selector_rows(x.data_ptr(), x.stride(0), rows, vocab, mode, temperature, scratch.data_ptr(),
                                 conf.data_ptr(), tok.data_ptr(), stream) == 0
    return conf, tok


def _no_alloc(lib, x, mode, temperature):
    rows, vocab = x.shape
    conf = torch.full((rows,), -1.0, dtype=torch.float64, device=x.device)
    tok = torch.full((rows,), -1, dtype=torch.int32, device=x.device)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.drt_selector_rows_noalloc(x.data_ptr(), x.stride(0), rows, vocab, mode, temperature, conf.data_ptr(),
                                       tok.data_ptr(), stream)
    assert rc == 0, lib.drt_last_error()
    return conf, tok


def test_noalloc_selector_matches_caller_scratch_selector(lib):
    from diffusorrt_b200 import _lib

    dev = torch.device("cuda:0")
    calls = [(32, 151936, _lib.SELECT_MAX_PROB, 0.0, 1), (9, 8195, _lib.SELECT_NEG_ENTROPY, 0.2, 2)]
    for rows, vocab, mode, temperature, seed in calls:
        x = torch.from_numpy(np.random.default_rng(seed).normal(0.0, 3.0, size=(rows, vocab)).astype(np.float32)).to(dev)
        want_conf, want_tok = _with_scratch(lib, x, mode, temperature)
        got_conf, got_tok = _no_alloc(lib, x, mode, temperature)
        torch.cuda.synchronize()
        assert got_tok.cpu().tolist() == want_tok.cpu().tolist()
        np.testing.assert_allclose(got_conf.cpu().numpy(), want_conf.cpu().numpy(), rtol=1e-13, atol=0)


def test_noalloc_selector_rejects_oversize_calls(lib):
    from diffusorrt_b200 import _lib

    rc = lib.drt_selector_rows_noalloc(ctypes.c_void_p(16), 200000, 1025, 151936, _lib.SELECT_MAX_PROB, 0.0,
                                       ctypes.c_void_p(16), ctypes.c_void_p(16), None)
    assert rc == _lib.INVALID_ARGUMENT
    assert b"at most 1024 rows" in lib.drt_last_error()
    rc = lib.drt_selector_rows_noalloc(ctypes.c_void_p(16), 300000, 1, 300000, _lib.SELECT_MAX_PROB, 0.0,
                                       ctypes.c_void_p(16), ctypes.c_void_p(16), None)
    assert rc == _lib.INVALID_ARGUMENT
