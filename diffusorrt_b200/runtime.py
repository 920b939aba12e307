"""Drop-in device-session provider for the DiffusorRT SDK's ``cuda_native`` route.

The SDK opens ``diffusorrt_runtime.Runtime(package_dir, device="cuda", engine_config=...,
precision=..., device_ordinal=..., creation_memory_budget_bytes=...)``
(python/src/edllm/model.py:873-920), then ``runtime.session(session_config)``
(model.py:1055-1067) and drives the session from ``generate_device_tokens`` /
``generate_window_tokens`` (python/src/edllm/backends/device_runtime.py:108-365):

    start_device(x, *, prompt_len, block_size, mask_token_id, exact_kv, steps,
                 memory_budget_bytes, temperature, seed)
    propose_device(frontier, *, window_end, frozen_prefix) -> (scores, token_ids, forwarded)
    commit_device(positions, token_ids)
    execute_window(token_ids, scope, *, mask_geometry=(prompt_len, block_size))
        -> .logits (LE f32 bytes [n_rows * n_vocab]), .n_rows, .n_vocab, .forwarded_rows
    device_metrics() -> dict

This module binds those calls to the native library (include/diffusorrt_b200.h) and adds
``Session.generate``: the whole request on the GPU (prefill, then CUDA-graph denoising steps
with plan / score / select / commit on the device), bit-compatible with driving the same
policy from the host through propose/commit.

Errors follow the reference boundary: contract violations raise ``ValueError``; unsupported
requests raise ``NotImplementedError``; device failures raise ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import json
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Mapping, Sequence

import numpy as np

from . import _lib
from .config import QWEN3_06B_BD3LM, SYNTHETIC_STD, rope_half_tables

_STRATEGY_IDS = {"block_threshold": _lib.STRATEGY_BLOCK_THRESHOLD, "bd3_fixed_quota": _lib.STRATEGY_BD3_FIXED_QUOTA,
                 "d2f_block_pipeline": _lib.STRATEGY_D2F_BLOCK_PIPELINE, "entropy_count": _lib.STRATEGY_ENTROPY_COUNT}
_COMMIT_IDS = {"threshold": _lib.COMMIT_THRESHOLD, "fixed_quota": _lib.COMMIT_FIXED_QUOTA}
_MASK_IDS = {"bidirectional": _lib.MASK_BIDIRECTIONAL, "d2f_hybrid": _lib.MASK_D2F_HYBRID}


class DeviceTimeout(RuntimeError):
    """A bounded device wait ran out (DRT_DEVICE_TIMEOUT): a tensor-parallel peer stopped, or a
    copy / MMA never completed. The session and the CUDA context stay usable."""


def _raise(exc: _lib.DrtError):
    if exc.status == _lib.INVALID_ARGUMENT:
        raise ValueError(str(exc)) from None
    if exc.status == _lib.UNSUPPORTED:
        raise NotImplementedError(str(exc)) from None
    if exc.status == _lib.DEVICE_TIMEOUT:
        raise DeviceTimeout(str(exc)) from None
    raise RuntimeError(str(exc)) from None


def _call(status: int) -> None:
    try:
        _lib.check(status)
    except _lib.DrtError as exc:
        _raise(exc)


@dataclass(frozen=True)
class WindowResult:
    """What ``execute_window`` returns (device_runtime.py:354-363)."""

    logits: bytes
    n_rows: int
    n_vocab: int
    forwarded_rows: int


def finalize(x: Sequence[int], prompt_len: int, mask_token_id: int, eos_token_id: int) -> dict:
    """The visible answer of a decoded canvas, as the reference's ``MaskState.finalize``
    (python/src/edllm/backends/diffusion_runtime.py:526-558): the answer ends at the first EOS of the
    generated region ("stop"); without EOS, or with masks left in the answer, the reason is
    "length"; the visible tokens end at the first unresolved (MASK) row."""
    gen = list(x[prompt_len:])
    if eos_token_id in gen:
        answer, hit_eos, reason = gen[:gen.index(eos_token_id)], True, "stop"
    else:
        answer, hit_eos, reason = gen, False, "length"
    remaining = answer.count(mask_token_id)
    if remaining:
        reason = "length"
        visible = answer[:answer.index(mask_token_id)]
    else:
        visible = answer
    return {"visible_token_ids": visible, "hit_eos": hit_eos, "remaining_mask_count": remaining,
            "finish_reason": reason}


def _as_int_list(values, name: str) -> list[int]:
    out = []
    for v in values:
        if isinstance(v, bool) or int(v) != v:
            raise ValueError(f"{name} must contain integers")
        out.append(int(v))
    return out


def _bf16_bits(array) -> np.ndarray:
    """uint16 bf16 encoding of an array: uint16 input is taken as bf16 bits, floats are rounded
    to nearest-even."""
    a = np.asarray(array)
    if a.dtype == np.uint16:
        return np.ascontiguousarray(a)
    if str(a.dtype) == "bfloat16":
        return np.ascontiguousarray(a.view(np.uint16))
    f = np.ascontiguousarray(a, dtype=np.float32)
    bits = f.view(np.uint32).astype(np.uint64)
    bits = (bits + np.uint64(0x7FFF) + ((bits >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    return bits.astype(np.uint16)


def _model_config(cfg: Mapping[str, Any], max_seq: int = 128, max_prefill_rows: int = 128) -> _lib.ModelConfig:
    return _lib.ModelConfig(
        layer_count=cfg["layer_count"], hidden_size=cfg["hidden_size"], attention_heads=cfg["attention_heads"],
        num_kv_heads=cfg["num_kv_heads"], head_dim=cfg["head_dim"], intermediate_size=cfg["intermediate_size"],
        vocab_size=cfg["vocab_size"], qk_norm=int(bool(cfg["qk_norm"])), qkv_bias=int(bool(cfg["qkv_bias"])),
        tied_lm_head=int(bool(cfg["tied_lm_head"])), rms_norm_eps=float(cfg["rms_norm_eps"]),
        rope_theta=float(cfg["rope_theta"]), max_seq=int(max_seq), max_prefill_rows=int(max_prefill_rows),
        logits_shift=int(bool(cfg.get("logits_shift", False))))


def tp_shard(lib, cfg: Mapping[str, Any], rank: int, world: int) -> dict:
    """Shard geometry of one tensor-parallel rank (host-only call into the library)."""
    out = _lib.TpShard()
    _call(lib.drt_tp_shard_geometry(ctypes.byref(_model_config(cfg)), int(rank), int(world), ctypes.byref(out)))
    return {name: getattr(out, name) for name, _ in _lib.TpShard._fields_}


def share_tp_id(rank: int, make_id) -> bytes:
    """Rank 0 makes the group's NCCL id; torch.distributed broadcasts it to every rank."""
    import torch.distributed as dist

    box = [make_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    nccl_id = box[0]
    if not isinstance(nccl_id, bytes) or len(nccl_id) != _lib.TP_ID_BYTES:
        raise RuntimeError("tensor-parallel id exchange failed")
    return nccl_id


class Runtime:
    """One model resident on one GPU (``diffusorrt_runtime.Runtime``); with
    ``tensor_parallel=True``, one rank's shard of a model split over a torch.distributed group."""

    def __init__(self, package_dir: str | Path | None = None, *, device: str = "cuda",
                 engine_config: Mapping[str, Any] | None = None, precision: Mapping[str, Any] | None = None,
                 device_ordinal: int = 0, creation_memory_budget_bytes: int = 0,
                 model_config: Mapping[str, Any] | None = None, weights: Mapping[str, Any] | None = None,
                 synthetic_seed: int | None = None, max_seq: int = 4608 + 128, max_prefill_rows: int = 4096,
                 tensor_parallel: bool = False):
        if device != "cuda":
            raise ValueError(f"this runtime serves device='cuda' only, not {device!r}")
        engine_config = dict(engine_config or {})
        if engine_config.get("compute_dtype", 0) not in (0, "bf16", "bfloat16"):
            raise NotImplementedError("the B200 engine computes with bf16 weights (compute_dtype 0)")
        quant_bits = engine_config.get("linear_quant_bits")
        quant_group = int(engine_config.get("linear_quant_group_size", 64) or 64)
        if quant_bits and (int(quant_bits) not in (4, 8) or quant_group != 64):
            raise NotImplementedError("linear quantization is served as 4-bit affine or int8, group size 64")
        if precision is not None:
            # cuda_precision_descriptor (python/src/edllm/backends/device_runtime.py:19-47): bf16, or the
            # int8_weight_only scheme (int8 weights, per-group scales of 64 inputs, bf16 activations)
            scheme = precision.get("scheme", "bf16")
            if scheme == "int8_weight_only" or precision.get("weight_type") == "int8":
                if precision.get("activation_type", "bf16") != "bf16" or precision.get("accumulation_type", "fp32") != "fp32":
                    raise NotImplementedError(f"precision {precision!r} is not served by this build")
                quant_bits = quant_bits or 8
                if int(quant_bits) != 8:
                    raise ValueError("the int8_weight_only precision quantizes linears to 8 bits")
            elif precision.get("weight_type", "bf16") != "bf16":
                raise NotImplementedError(f"precision {scheme!r} is not served by this build")
        cfg = dict(QWEN3_06B_BD3LM)
        package = None
        if package_dir is not None:
            meta = Path(package_dir) / "model.json"
            if meta.exists():
                doc = json.loads(meta.read_text())
                if doc.get("package_format") is not None:
                    # a converted package: geometry from its GraphIR and tensors, weights from its
                    # verified safetensors shards (package.py)
                    from .package import read_package

                    package = read_package(package_dir)
                    cfg.update(package.config)
                else:
                    cfg.update({k: v for k, v in doc.get("runtime_config", doc).items() if k in cfg})
                    if synthetic_seed is None and "synthetic_seed" in doc:
                        synthetic_seed = int(doc["synthetic_seed"])
        if model_config:
            cfg.update(model_config)
        self.config = cfg
        self.device_ordinal = int(device_ordinal)
        self._lib = _lib.load()
        mc = _model_config(cfg, max_seq, max_prefill_rows)
        handle = ctypes.c_void_p()
        self.tp_rank, self.tp_world = 0, 1
        if tensor_parallel:
            # one rank of a tensor-parallel group: torch.distributed (already initialised, one
            # process per GPU) carries the NCCL id; the model joins the group's communicator
            import torch.distributed as dist

            self.tp_rank, self.tp_world = dist.get_rank(), dist.get_world_size()
            nccl_id = share_tp_id(self.tp_rank, self._make_tp_id)
            _call(self._lib.drt_model_create_tp(ctypes.byref(mc), self.device_ordinal, self.tp_rank, self.tp_world,
                                                nccl_id, ctypes.byref(handle)))
        else:
            _call(self._lib.drt_model_create(ctypes.byref(mc), self.device_ordinal, ctypes.byref(handle)))
        self._model = handle
        self.max_seq = int(max_seq)
        cos, sin = rope_half_tables(self.max_seq, cfg["head_dim"], float(cfg["rope_theta"]))
        _call(self._lib.drt_model_set_rope(self._model, cos.ctypes.data, sin.ctypes.data, self.max_seq))
        self.quantized = False
        self.package = package
        if synthetic_seed is not None:
            self.init_synthetic(synthetic_seed)
        if package is not None:
            self.load_package(package)
        if weights is not None:
            self.load_weights(weights)
        if quant_bits:
            self.quantize(int(quant_bits), quant_group)
        if creation_memory_budget_bytes and self.device_bytes > int(creation_memory_budget_bytes):
            self.close()
            raise ValueError("model weights exceed creation_memory_budget_bytes")

    def _make_tp_id(self) -> bytes:
        buf = ctypes.create_string_buffer(_lib.TP_ID_BYTES)
        _call(self._lib.drt_tp_unique_id(buf))
        return buf.raw

    def shard(self) -> dict:
        """This rank's shard geometry (the whole model for a single GPU)."""
        return tp_shard(self._lib, self.config, self.tp_rank, self.tp_world)

    # ------------------------------------------------------------------ weights
    def init_synthetic(self, seed: int, *, linear_std: float | None = None, embed_std: float | None = None,
                       bias_std: float | None = None) -> None:
        std = dict(SYNTHETIC_STD)
        for k, v in (("linear_std", linear_std), ("embed_std", embed_std), ("bias_std", bias_std)):
            if v is not None:
                std[k] = v
        _call(self._lib.drt_model_init_synthetic(self._model, int(seed) & (2**64 - 1), std["linear_std"],
                                                 std["embed_std"], std["bias_std"]))
        if getattr(self, "quantized", False):
            self.quantize()

    def load_weights(self, weights: Mapping[str, Any]) -> None:
        """Install tensors by package key (``model.layers.N.self_attn.q_proj.weight`` ...)."""
        for key, value in weights.items():
            if key == "lm_head.weight" and self.config["tied_lm_head"]:
                continue
            arr = np.asarray(value)
            rows = arr.shape[0] if arr.ndim == 2 else 1
            cols = arr.shape[-1]
            if arr.ndim == 1 or key.endswith("norm.weight") or key.endswith(".bias"):
                data = np.ascontiguousarray(arr, dtype=np.float32)
                _call(self._lib.drt_model_set_tensor(self._model, key.encode(), data.ctypes.data, 1, rows, cols))
            else:
                data = _bf16_bits(arr)
                _call(self._lib.drt_model_set_tensor(self._model, key.encode(), data.ctypes.data, 0, rows, cols))
        if getattr(self, "quantized", False):
            self.quantize()

    def load_package(self, package) -> None:
        """Install every tensor of a verified package (``package.read_package``) as stored: bf16
        matrices as their bits, bf16 vectors (norms, biases) widened exactly to float32."""
        for name, arr in package.items():
            if name == "lm_head.weight" and self.config["tied_lm_head"]:
                continue
            rows = arr.shape[0] if arr.ndim == 2 else 1
            cols = arr.shape[-1]
            if arr.dtype == np.uint16:  # bf16 bits
                data = np.ascontiguousarray(arr)
                _call(self._lib.drt_model_set_tensor(self._model, name.encode(), data.ctypes.data, 0, rows, cols))
            elif arr.ndim == 1:
                data = np.ascontiguousarray(arr, dtype=np.float32)
                _call(self._lib.drt_model_set_tensor(self._model, name.encode(), data.ctypes.data, 1, rows, cols))
            else:
                data = _bf16_bits(np.asarray(arr, dtype=np.float32))
                _call(self._lib.drt_model_set_tensor(self._model, name.encode(), data.ctypes.data, 0, rows, cols))
        if getattr(self, "quantized", False):
            self.quantize()

    def quantize(self, bits: int | None = None, group_size: int = 64) -> None:
        """Quantized copies of every layer linear and lm_head, later forwards use them: 4-bit affine
        (the reference's load-time ``_quantize_linear_weights``, mlx_dream.py:2090-2108) or 8 (the
        CUDA ``int8_weight_only`` precision). By default the width of the model's last quantization
        (4 for a first one)."""
        bits = int(bits if bits is not None else getattr(self, "quant_bits", 4))
        _call(self._lib.drt_model_quantize(self._model, bits, int(group_size)))
        self.quantized = True
        self.quant_bits = bits

    def get_tensor(self, key: str, shape: tuple[int, int]) -> np.ndarray:
        """A resident tensor as float32 (bf16 values widened)."""
        out = np.empty(shape, dtype=np.float32)
        _call(self._lib.drt_model_get_tensor(self._model, key.encode(), out.ctypes.data, 1, shape[0], shape[1]))
        return out

    @property
    def device_bytes(self) -> int:
        return int(self._lib.drt_model_device_bytes(self._model))

    # ------------------------------------------------------------------ sessions
    def session(self, session_config: Mapping[str, Any] | None = None) -> "Session":
        return Session(self, dict(session_config or {}))

    def close(self) -> None:
        if getattr(self, "_model", None):
            self._lib.drt_model_destroy(self._model)
            self._model = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass


def _enum(value, table: dict, name: str) -> int:
    if isinstance(value, str):
        if value not in table:
            raise ValueError(f"{name}={value!r} is not served by this device session")
        return table[value]
    if int(value) not in table.values():
        raise ValueError(f"{name}={value!r} is not served by this device session")
    return int(value)


class Session:
    """One decode request's device state (K/V cache, canvas, graphs). Single-threaded."""

    def __init__(self, runtime: Runtime, session_config: dict):
        self.runtime = runtime
        self._lib = runtime._lib
        strategy = _enum(session_config.get("decode_strategy", "bd3_fixed_quota"), _STRATEGY_IDS, "decode_strategy")
        default_commit = ("threshold" if strategy in (_lib.STRATEGY_BLOCK_THRESHOLD, _lib.STRATEGY_D2F_BLOCK_PIPELINE)
                          else "fixed_quota")
        commit = _enum(session_config.get("commit_policy", default_commit), _COMMIT_IDS, "commit_policy")
        default_mask = "bidirectional" if strategy == _lib.STRATEGY_ENTROPY_COUNT else "d2f_hybrid"
        mask = _enum(session_config.get("attention_mask_kind", default_mask), _MASK_IDS, "attention_mask_kind")
        self.block_size = int(session_config.get("block_size", runtime.config.get("block_size", 32)))
        sc = _lib.SessionConfig(decode_strategy=strategy, commit_policy=commit, attention_mask_kind=mask,
                                block_size=self.block_size, steps=int(session_config.get("steps", 128)),
                                max_tokens=int(session_config.get("max_tokens", 0)))
        handle = ctypes.c_void_p()
        _call(self._lib.drt_session_open(runtime._model, ctypes.byref(sc), ctypes.byref(handle)))
        self._s = handle
        self.decode_strategy = strategy
        self.vocab = int(runtime.config["vocab_size"])
        if runtime.tp_world > 1 and session_config.get("tp_peer_memory", True):
            # map every rank's partial-sum buffer (collective: every rank opens its session in turn)
            import torch.distributed as dist

            buf = ctypes.create_string_buffer(_lib.TP_HANDLE_BYTES)
            _call(self._lib.drt_session_tp_handle(self._s, buf))
            handles = [None] * runtime.tp_world
            dist.all_gather_object(handles, buf.raw)
            _call(self._lib.drt_session_tp_connect(self._s, b"".join(handles), runtime.tp_world))
            if not session_config.get("tp_vocab_parallel", True):
                # every rank projects the whole vocabulary (the default splits the lm_head by vocabulary)
                _call(self._lib.drt_session_tp_vocab_parallel(self._s, 0))

    # ------------------------------------------------------------------ reference surface
    def start_device(self, x: Sequence[int], *, prompt_len: int, block_size: int, mask_token_id: int,
                     exact_kv: bool, steps: int, memory_budget_bytes: int = 0, temperature: float = 0.0,
                     seed: int = 0) -> None:
        ids = _as_int_list(x, "x")
        arr = _lib.i32_array(ids)
        _call(self._lib.drt_session_start(self._s, arr, len(ids), int(prompt_len), int(block_size),
                                          int(mask_token_id), int(bool(exact_kv)), int(steps),
                                          int(memory_budget_bytes), float(temperature), int(seed) & (2**64 - 1)))

    def propose_device(self, frontier: Sequence[int], *, window_end: int, frozen_prefix: int):
        fr = _as_int_list(frontier, "frontier")
        n = len(fr)
        scores = (ctypes.c_double * max(1, n))()
        tokens = (ctypes.c_int32 * max(1, n))()
        forwarded = ctypes.c_int32()
        _call(self._lib.drt_session_propose(self._s, _lib.i32_array(fr), n, int(window_end), int(frozen_prefix),
                                            scores, tokens, ctypes.byref(forwarded)))
        return [float(scores[i]) for i in range(n)], [int(tokens[i]) for i in range(n)], int(forwarded.value)

    def commit_device(self, positions: Sequence[int], token_ids: Sequence[int]) -> None:
        pos = _as_int_list(positions, "positions")
        tok = _as_int_list(token_ids, "token_ids")
        if len(pos) != len(tok):
            raise ValueError("commit positions and token ids differ in length")
        _call(self._lib.drt_session_commit(self._s, _lib.i32_array(pos), _lib.i32_array(tok), len(pos)))

    def execute_window(self, token_ids: Sequence[int], scope: Sequence[int], *, mask_geometry=None) -> WindowResult:
        ids = _as_int_list(token_ids, "token_ids")
        sc = _as_int_list(scope, "scope")
        if mask_geometry is None:
            if self.decode_strategy != _lib.STRATEGY_ENTROPY_COUNT:
                raise NotImplementedError("this device session executes d2f_hybrid windows; pass mask_geometry")
            mask_geometry = (0, 1)  # bidirectional: the geometry is unused
        prompt_len, block_size = (int(v) for v in mask_geometry)
        out = np.empty((len(sc), self.vocab), dtype="<f4")
        forwarded = ctypes.c_int32()
        _call(self._lib.drt_session_execute_window(self._s, _lib.i32_array(ids), len(ids), _lib.i32_array(sc), len(sc),
                                                   prompt_len, block_size, out.ctypes.data, ctypes.byref(forwarded)))
        return WindowResult(logits=out.tobytes(), n_rows=len(sc), n_vocab=self.vocab,
                            forwarded_rows=int(forwarded.value))

    def device_metrics(self) -> dict:
        m = _lib.Metrics()
        _call(self._lib.drt_session_metrics(self._s, ctypes.byref(m)))
        return {name: getattr(m, name) for name, _ in _lib.Metrics._fields_}

    # ------------------------------------------------------------------ device-resident request
    def generate(self, prompt: Sequence[int], *, max_tokens: int, steps: int, block_size: int | None = None,
                 decode_strategy: str | None = None, mask_token_id: int | None = None,
                 eos_token_id: int | None = None, confidence_threshold: float = 0.9, rounds_per_block: int = 0,
                 trace_steps: int = 0, temperature: float | None = None, top_p: float | None = 0.95,
                 eps: float = 1e-3, seed: int = 0, mask_origin: int | str | None = None,
                 add_threshold: float = 0.1, activate_threshold: float = 0.95) -> dict:
        """Whole request on the device. ``decode_strategy="entropy_count"`` (a session opened with
        that strategy) runs the Dream full-canvas schedule with NegEntropy(temperature, top_p) and
        linspace(1, eps, steps + 1) timesteps (temperature defaults to 0.2); the others run the BD3 /
        block-threshold loops, where ``temperature`` > 0 (bd3_fixed_quota only) draws each row's token
        keyed by ``seed`` (default 0: argmax). ``mask_origin`` is the d2f mask geometry's origin: 0
        for the BD3LM graph's absolute blocks, ``"prompt"`` for the Dream D2F graph (prompt
        bidirectional, blocks counted from it); by default the model config's ``mask_origin`` (0).
        The result carries the final canvas ``x`` and the reference's finalize fields
        (``visible_token_ids``, ``hit_eos``, ``remaining_mask_count``, ``finish_reason``)."""
        cfg = self.runtime.config
        ids = _as_int_list(prompt, "prompt")
        strategy = self.decode_strategy if decode_strategy is None else _enum(decode_strategy, _STRATEGY_IDS,
                                                                             "decode_strategy")
        if temperature is None:
            temperature = 0.2 if strategy == _lib.STRATEGY_ENTROPY_COUNT else 0.0
        if mask_origin is None:
            mask_origin = cfg.get("mask_origin", 0)
        origin = -1 if mask_origin == "prompt" else int(mask_origin)
        mask_id = int(cfg["mask_token_id"] if mask_token_id is None else mask_token_id)
        eos_id = int(cfg["eos_token_id"] if eos_token_id is None else eos_token_id)
        params = _lib.GenerateParams(
            decode_strategy=strategy, steps=int(steps),
            block_size=int(block_size or self.block_size), max_tokens=int(max_tokens),
            mask_token_id=mask_id, eos_token_id=eos_id,
            confidence_threshold=float(confidence_threshold), rounds_per_block=int(rounds_per_block),
            trace_steps=int(trace_steps), temperature=float(temperature),
            top_p=1.0 if top_p is None else float(top_p), eps=float(eps), seed=int(seed) & (2**64 - 1),
            mask_origin=origin, add_threshold=float(add_threshold), activate_threshold=float(activate_threshold))
        out = (ctypes.c_int32 * (len(ids) + int(max_tokens)))()
        res = _lib.GenerateResult()
        trace = (_lib.StepTrace * max(1, int(trace_steps)))() if trace_steps else None
        _call(self._lib.drt_session_generate(self._s, ctypes.byref(params), _lib.i32_array(ids), len(ids), out,
                                             ctypes.byref(res), trace))
        result = {name: getattr(res, name) for name, _ in _lib.GenerateResult._fields_}
        result["x"] = list(out)
        result.update(finalize(result["x"], len(ids), mask_id, eos_id))
        if trace is not None:
            steps_out = []
            for t in trace[: min(res.forward_count, int(trace_steps))]:
                n = t.n_frontier
                steps_out.append({"step": t.step, "frontier": list(t.frontier_pos[:n]), "tokens": list(t.token[:n]),
                                  "scores": list(t.conf[:n]), "tie": t.tie,
                                  "chosen": [i for i in range(n) if (t.chosen_mask >> i) & 1]})
            result["trace"] = steps_out
        return result

    def peer_wait_drill(self) -> None:
        """Run one bounded peer-flag wait that nothing satisfies (drt_session_peer_wait_drill);
        raises DeviceTimeout after the wait limit, leaving the session usable."""
        _call(self._lib.drt_session_peer_wait_drill(self._s))

    def kv_pointers(self) -> tuple[int, int]:
        k, v = ctypes.c_void_p(), ctypes.c_void_p()
        _call(self._lib.drt_session_kv_pointers(self._s, ctypes.byref(k), ctypes.byref(v)))
        return int(k.value or 0), int(v.value or 0)

    def close(self) -> None:
        if getattr(self, "_s", None):
            self._lib.drt_session_close(self._s)
            self._s = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass
