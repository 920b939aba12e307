"""Kernel-level entry points on torch CUDA tensors (device memory and streams come from torch).

These call the C ABI directly with device pointers; they are the unit-level surface used by the
selector microbenchmark and the kernel parity tests.
"""
from __future__ import annotations

import torch

from . import _lib


def _stream_ptr(stream: torch.cuda.Stream | None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def selector_scratch(n_rows: int, vocab: int, device) -> torch.Tensor:
    nbytes = int(_lib.load().drt_selector_scratch_bytes(int(n_rows), int(vocab)))
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def select_rows(logits: torch.Tensor, *, mode: int = _lib.SELECT_MAX_PROB, temperature: float = 0.0,
                scratch: torch.Tensor | None = None, conf: torch.Tensor | None = None,
                token: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None):
    """Per-row (confidence f64, token i32) of f32 logits [rows, vocab] (row stride may exceed vocab)."""
    if logits.dtype != torch.float32 or not logits.is_cuda or logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a row-major CUDA float32 [rows, vocab] tensor")
    rows, vocab = logits.shape
    dev = logits.device
    if scratch is None:
        scratch = selector_scratch(rows, vocab, dev)
    if conf is None:
        conf = torch.empty(rows, dtype=torch.float64, device=dev)
    if token is None:
        token = torch.empty(rows, dtype=torch.int32, device=dev)
    _lib.check(_lib.load().drt_selector_rows(logits.data_ptr(), logits.stride(0), rows, vocab, int(mode),
                                             float(temperature), scratch.data_ptr(), conf.data_ptr(),
                                             token.data_ptr(), _stream_ptr(stream)))
    return conf, token


def select_sample(logits: torch.Tensor, positions: torch.Tensor, *, temperature: float, seed: int, forward: int,
                  row_index: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None):
    """Temperature-sampled (confidence f64, token i32, tie i32) per row of f32 logits [rows, vocab]
    (or of the rows row_index), keyed by (seed, forward, positions[r]) as drt_selector_sample."""
    if logits.dtype != torch.float32 or not logits.is_cuda or logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a row-major CUDA float32 [rows, vocab] tensor")
    if positions.dtype != torch.int32 or not positions.is_cuda or not positions.is_contiguous():
        raise ValueError("positions must be a contiguous CUDA int32 tensor")
    n = positions.numel() if row_index is None else row_index.numel()
    if row_index is None and n != logits.shape[0]:
        raise ValueError("one position per logits row")
    vocab = logits.shape[1]
    dev = logits.device
    scratch = selector_scratch(n, vocab, dev)
    conf = torch.empty(n, dtype=torch.float64, device=dev)
    token = torch.empty(n, dtype=torch.int32, device=dev)
    tie = torch.empty(n, dtype=torch.int32, device=dev)
    _lib.check(_lib.load().drt_selector_sample(logits.data_ptr(), logits.stride(0),
                                               0 if row_index is None else row_index.data_ptr(), n, vocab,
                                               float(temperature), int(seed) & (2**64 - 1), int(forward),
                                               positions.data_ptr(), scratch.data_ptr(), conf.data_ptr(),
                                               token.data_ptr(), tie.data_ptr(), _stream_ptr(stream)))
    return conf, token, tie


CHOICE_TOPK = 0
CHOICE_THRESHOLD = 1


def select_gather(logits: torch.Tensor, row_index: torch.Tensor, *, mode: int = _lib.SELECT_MAX_PROB,
                  temperature: float = 0.0, scratch: torch.Tensor | None = None, conf: torch.Tensor | None = None,
                  token: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None):
    """(confidence f64, token i32) for the rows row_index (int32 CUDA) of f32 logits [rows, vocab]."""
    if logits.dtype != torch.float32 or not logits.is_cuda or logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a row-major CUDA float32 [rows, vocab] tensor")
    if row_index.dtype != torch.int32 or not row_index.is_cuda or not row_index.is_contiguous():
        raise ValueError("row_index must be a contiguous CUDA int32 tensor")
    n = row_index.numel()
    vocab = logits.shape[1]
    dev = logits.device
    if scratch is None:
        scratch = selector_scratch(n, vocab, dev)
    if conf is None:
        conf = torch.empty(n, dtype=torch.float64, device=dev)
    if token is None:
        token = torch.empty(n, dtype=torch.int32, device=dev)
    _lib.check(_lib.load().drt_selector_gather(logits.data_ptr(), logits.stride(0), row_index.data_ptr(), n, vocab,
                                               int(mode), float(temperature), scratch.data_ptr(), conf.data_ptr(),
                                               token.data_ptr(), _stream_ptr(stream)))
    return conf, token


def select_topp_entropy(logits: torch.Tensor, row_index: torch.Tensor | None = None, *, temperature: float = 0.2,
                        top_p: float = 0.95, exclude_token: int = -1, tie_rel: float = 2.0 ** -30,
                        stream: torch.cuda.Stream | None = None):
    """NegEntropy with a top-p nucleus over rows (row_index, int32 CUDA, or every row) of f32 logits:
    (confidence f64 holding the f32 value, token i32, tie bits i32)."""
    if logits.dtype != torch.float32 or not logits.is_cuda or logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a row-major CUDA float32 [rows, vocab] tensor")
    if row_index is not None and (row_index.dtype != torch.int32 or not row_index.is_contiguous()):
        raise ValueError("row_index must be a contiguous CUDA int32 tensor")
    n = row_index.numel() if row_index is not None else logits.shape[0]
    dev = logits.device
    conf = torch.empty(n, dtype=torch.float64, device=dev)
    token = torch.empty(n, dtype=torch.int32, device=dev)
    tie = torch.empty(max(1, n), dtype=torch.int32, device=dev)
    _lib.check(_lib.load().drt_selector_topp(logits.data_ptr(), logits.stride(0),
                                             row_index.data_ptr() if row_index is not None else None, n,
                                             logits.shape[1], float(temperature), float(top_p), int(exclude_token),
                                             float(tie_rel), conf.data_ptr(), token.data_ptr(), tie.data_ptr(),
                                             _stream_ptr(stream)))
    return conf, token, tie[:n]


def select_choices(conf: torch.Tensor, offsets: torch.Tensor, *, mode: int, k: int = 1, tau: float = 0.9,
                   tie_rel: float = 2.0 ** -40, chosen: torch.Tensor | None = None, tie: torch.Tensor | None = None,
                   stream: torch.cuda.Stream | None = None):
    """Top-k (mode CHOICE_TOPK) or threshold (CHOICE_THRESHOLD) choices per confidence run
    offsets[b] .. offsets[b + 1]: chosen[row] in {0, 1} (int32) and tie[b] certification bits."""
    if conf.dtype != torch.float64 or offsets.dtype != torch.int32:
        raise ValueError("conf must be float64 and offsets int32 CUDA tensors")
    n_items = offsets.numel() - 1
    if chosen is None:
        chosen = torch.empty(conf.numel(), dtype=torch.int32, device=conf.device)
    if tie is None:
        tie = torch.empty(max(1, n_items), dtype=torch.int32, device=conf.device)
    _lib.check(_lib.load().drt_select_choices(conf.data_ptr(), offsets.data_ptr(), n_items, int(mode), int(k),
                                              float(tau), float(tie_rel), chosen.data_ptr(), tie.data_ptr(),
                                              _stream_ptr(stream)))
    return chosen, tie


def linear_bf16(x: torch.Tensor, w: torch.Tensor, *, splits: int = 1, round_bf16: bool = True,
                out: torch.Tensor | None = None, scratch: torch.Tensor | None = None,
                stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """y = x @ w^T on the tcgen05 path: x [rows, K] bf16, w [n, K] bf16 -> y [rows, n] f32."""
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or not x.is_contiguous() or not w.is_contiguous():
        raise ValueError("x and w must be contiguous bf16 CUDA tensors")
    rows, K = x.shape
    n = w.shape[0]
    if out is None:
        out = torch.empty(rows, n, dtype=torch.float32, device=x.device)
    lib = _lib.load()
    if scratch is None:
        scratch = torch.empty(int(lib.drt_linear_scratch_bytes(rows, n, K, splits)), dtype=torch.uint8, device=x.device)
    _lib.check(lib.drt_linear_bf16(x.data_ptr(), w.data_ptr(), out.data_ptr(), rows, n, K, int(splits),
                                   int(bool(round_bf16)), scratch.data_ptr(), _stream_ptr(stream)))
    return out


def quantize_q4(w: torch.Tensor, *, stream: torch.cuda.Stream | None = None):
    """4-bit affine quantization of a bf16 [rows, K] weight: (packed uint8 [rows, K/2],
    scale bf16 [rows, K/64], bias bf16 [rows, K/64])."""
    if w.dtype != torch.bfloat16 or not w.is_contiguous() or w.dim() != 2:
        raise ValueError("w must be a contiguous bf16 CUDA matrix")
    rows, K = w.shape
    q = torch.empty(rows, K // 2, dtype=torch.uint8, device=w.device)
    scale = torch.empty(rows, K // 64, dtype=torch.bfloat16, device=w.device)
    bias = torch.empty(rows, K // 64, dtype=torch.bfloat16, device=w.device)
    _lib.check(_lib.load().drt_quantize_q4(w.data_ptr(), rows, K, q.data_ptr(), scale.data_ptr(), bias.data_ptr(),
                                           _stream_ptr(stream)))
    return q, scale, bias


def quantize_q8(w: torch.Tensor, *, stream: torch.cuda.Stream | None = None):
    """int8 weight-only quantization of a bf16 [rows, K] weight: (bytes uint8 [rows, K] = q + 128,
    scale bf16 [rows, K/64], bias = -128 * scale bf16 [rows, K/64])."""
    if w.dtype != torch.bfloat16 or not w.is_contiguous() or w.dim() != 2:
        raise ValueError("w must be a contiguous bf16 CUDA matrix")
    rows, K = w.shape
    q = torch.empty(rows, K, dtype=torch.uint8, device=w.device)
    scale = torch.empty(rows, K // 64, dtype=torch.bfloat16, device=w.device)
    bias = torch.empty(rows, K // 64, dtype=torch.bfloat16, device=w.device)
    _lib.check(_lib.load().drt_quantize_q8(w.data_ptr(), rows, K, q.data_ptr(), scale.data_ptr(), bias.data_ptr(),
                                           _stream_ptr(stream)))
    return q, scale, bias


def linear_q8(x: torch.Tensor, q: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor, *, splits: int = 1,
              out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """y = bf16(x @ dequant(q, scale, bias)^T) widened to f32 (int8 weight-only): x [rows <= 64, K] bf16."""
    rows, K = x.shape
    n = q.shape[0]
    if out is None:
        out = torch.empty(rows, n, dtype=torch.float32, device=x.device)
    _lib.check(_lib.load().drt_linear_q8(x.data_ptr(), q.data_ptr(), scale.data_ptr(), bias.data_ptr(), out.data_ptr(),
                                         rows, n, K, int(splits), _stream_ptr(stream)))
    return out


def linear_q4(x: torch.Tensor, q: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor, *, splits: int = 1,
              out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """y = x @ dequant(q, scale, bias)^T (f32, no output rounding): x [rows <= 64, K] bf16."""
    rows, K = x.shape
    n = q.shape[0]
    if out is None:
        out = torch.empty(rows, n, dtype=torch.float32, device=x.device)
    _lib.check(_lib.load().drt_linear_q4(x.data_ptr(), q.data_ptr(), scale.data_ptr(), bias.data_ptr(), out.data_ptr(),
                                         rows, n, K, int(splits), _stream_ptr(stream)))
    return out
