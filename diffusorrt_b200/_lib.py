"""ctypes binding of libdiffusorrt_b200.so (the C ABI declared in include/diffusorrt_b200.h).

The shared library is built in-tree by ``diffusorrt_b200.build``. There is no fallback: if the
library is missing or a call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_NAME = "libdiffusorrt_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

# drt_status (AbiStatus values of python/src/edllm/abi/forward.py:20-25, plus one).
OK = 0
VERSION_MISMATCH = 1
INVALID_ARGUMENT = 2
UNSUPPORTED = 3
INTERNAL_ERROR = 4
DEVICE_TIMEOUT = 5
STATUS_NAMES = {0: "OK", 1: "VERSION_MISMATCH", 2: "INVALID_ARGUMENT", 3: "UNSUPPORTED", 4: "INTERNAL_ERROR",
                5: "DEVICE_TIMEOUT"}

STRATEGY_BLOCK_THRESHOLD = 0
STRATEGY_D2F_BLOCK_PIPELINE = 2
STRATEGY_ENTROPY_COUNT = 5
STRATEGY_BD3_FIXED_QUOTA = 7
COMMIT_THRESHOLD = 2
COMMIT_FIXED_QUOTA = 3
MASK_BIDIRECTIONAL = 0
MASK_D2F_HYBRID = 1
SELECT_MAX_PROB = 0
SELECT_NEG_ENTROPY = 1
TIE_NEAR = 1
TIE_EXACT = 2


class DrtError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class ModelConfig(ctypes.Structure):
    _fields_ = [("layer_count", ctypes.c_int32), ("hidden_size", ctypes.c_int32), ("attention_heads", ctypes.c_int32),
                ("num_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("intermediate_size", ctypes.c_int32),
                ("vocab_size", ctypes.c_int32), ("qk_norm", ctypes.c_int32), ("qkv_bias", ctypes.c_int32),
                ("tied_lm_head", ctypes.c_int32), ("rms_norm_eps", ctypes.c_float), ("rope_theta", ctypes.c_float),
                ("max_seq", ctypes.c_int32), ("max_prefill_rows", ctypes.c_int32), ("logits_shift", ctypes.c_int32)]


class TpShard(ctypes.Structure):
    _fields_ = [("rank", ctypes.c_int32), ("world", ctypes.c_int32), ("q_head0", ctypes.c_int32),
                ("q_heads", ctypes.c_int32), ("kv_head0", ctypes.c_int32), ("kv_heads", ctypes.c_int32),
                ("inter0", ctypes.c_int32), ("inter", ctypes.c_int32)]


TP_ID_BYTES = 128
TP_HANDLE_BYTES = 64


class SessionConfig(ctypes.Structure):
    _fields_ = [("decode_strategy", ctypes.c_int32), ("commit_policy", ctypes.c_int32),
                ("attention_mask_kind", ctypes.c_int32), ("block_size", ctypes.c_int32), ("steps", ctypes.c_int32),
                ("max_tokens", ctypes.c_int32)]


class GenerateParams(ctypes.Structure):
    _fields_ = [("decode_strategy", ctypes.c_int32), ("steps", ctypes.c_int32), ("block_size", ctypes.c_int32),
                ("max_tokens", ctypes.c_int32), ("mask_token_id", ctypes.c_int32), ("eos_token_id", ctypes.c_int32),
                ("confidence_threshold", ctypes.c_double), ("rounds_per_block", ctypes.c_int32),
                ("trace_steps", ctypes.c_int32), ("temperature", ctypes.c_double), ("top_p", ctypes.c_double),
                ("eps", ctypes.c_double), ("seed", ctypes.c_uint64), ("mask_origin", ctypes.c_int32),
                ("add_threshold", ctypes.c_double), ("activate_threshold", ctypes.c_double)]


class GenerateResult(ctypes.Structure):
    _fields_ = [("forward_count", ctypes.c_int32), ("iteration_count", ctypes.c_int32),
                ("committed_token_count", ctypes.c_int32), ("near_tie_steps", ctypes.c_int32),
                ("exact_tie_steps", ctypes.c_int32), ("stopped", ctypes.c_int32), ("canvas_len", ctypes.c_int32),
                ("prefill_ms", ctypes.c_float), ("decode_ms", ctypes.c_float), ("total_ms", ctypes.c_float),
                ("kernel_launches", ctypes.c_int32), ("host_enqueue_ms", ctypes.c_float)]


class StepTrace(ctypes.Structure):
    _fields_ = [("step", ctypes.c_int32), ("n_frontier", ctypes.c_int32), ("n_chosen", ctypes.c_int32),
                ("tie", ctypes.c_int32), ("frontier_pos", ctypes.c_int32 * 64), ("token", ctypes.c_int32 * 64),
                ("conf", ctypes.c_double * 64), ("chosen_mask", ctypes.c_uint64)]


class Metrics(ctypes.Structure):
    _fields_ = [("forward_count", ctypes.c_int64), ("forwarded_rows", ctypes.c_int64), ("prefill_rows", ctypes.c_int64),
                ("committed_token_count", ctypes.c_int64), ("near_tie_steps", ctypes.c_int64),
                ("exact_tie_steps", ctypes.c_int64), ("forward_ms_total", ctypes.c_double),
                ("device_bytes", ctypes.c_int64)]


_P = ctypes.c_void_p
_I32P = ctypes.POINTER(ctypes.c_int32)
_F64P = ctypes.POINTER(ctypes.c_double)

# name -> (restype, argtypes); every function declared in include/diffusorrt_b200.h.
SIGNATURES = {
    "drt_abi_version": (ctypes.c_int, [_I32P, _I32P, _I32P]),
    "drt_last_error": (ctypes.c_char_p, []),
    "drt_device_count": (ctypes.c_int, [_I32P]),
    "drt_model_create": (ctypes.c_int, [ctypes.POINTER(ModelConfig), ctypes.c_int32, ctypes.POINTER(_P)]),
    "drt_model_init_synthetic": (ctypes.c_int, [_P, ctypes.c_uint64, ctypes.c_float, ctypes.c_float, ctypes.c_float]),
    "drt_model_set_tensor": (ctypes.c_int, [_P, ctypes.c_char_p, _P, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64]),
    "drt_model_get_tensor": (ctypes.c_int, [_P, ctypes.c_char_p, _P, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64]),
    "drt_model_set_rope": (ctypes.c_int, [_P, _P, _P, ctypes.c_int32]),
    "drt_model_device_bytes": (ctypes.c_int64, [_P]),
    "drt_model_destroy": (None, [_P]),
    "drt_tp_shard_geometry": (ctypes.c_int, [ctypes.POINTER(ModelConfig), ctypes.c_int32, ctypes.c_int32,
                                             ctypes.POINTER(TpShard)]),
    "drt_tp_unique_id": (ctypes.c_int, [ctypes.c_char_p]),
    "drt_tp_flag_value": (ctypes.c_uint64, [ctypes.c_uint64, ctypes.c_int32, ctypes.c_int32]),
    "drt_model_create_tp": (ctypes.c_int, [ctypes.POINTER(ModelConfig), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                           ctypes.c_char_p, ctypes.POINTER(_P)]),
    "drt_model_quantize": (ctypes.c_int, [_P, ctypes.c_int32, ctypes.c_int32]),
    "drt_session_open": (ctypes.c_int, [_P, ctypes.POINTER(SessionConfig), ctypes.POINTER(_P)]),
    "drt_session_start": (ctypes.c_int, [_P, _I32P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                         ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, ctypes.c_double,
                                         ctypes.c_uint64]),
    "drt_session_propose": (ctypes.c_int, [_P, _I32P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _F64P, _I32P,
                                           _I32P]),
    "drt_session_commit": (ctypes.c_int, [_P, _I32P, _I32P, ctypes.c_int32]),
    "drt_session_execute_window": (ctypes.c_int, [_P, _I32P, ctypes.c_int32, _I32P, ctypes.c_int32, ctypes.c_int32,
                                                  ctypes.c_int32, _P, _I32P]),
    "drt_session_generate": (ctypes.c_int, [_P, ctypes.POINTER(GenerateParams), _I32P, ctypes.c_int32, _I32P,
                                            ctypes.POINTER(GenerateResult), ctypes.POINTER(StepTrace)]),
    "drt_session_metrics": (ctypes.c_int, [_P, ctypes.POINTER(Metrics)]),
    "drt_session_tp_handle": (ctypes.c_int, [_P, ctypes.c_char_p]),
    "drt_session_tp_connect": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.c_int32]),
    "drt_session_tp_vocab_parallel": (ctypes.c_int, [_P, ctypes.c_int32]),
    "drt_session_peer_wait_drill": (ctypes.c_int, [_P]),
    "drt_entropy_count_schedule": (ctypes.c_int, [ctypes.c_int32, ctypes.c_int32, ctypes.c_double, _I32P]),
    "drt_session_kv_pointers": (ctypes.c_int, [_P, ctypes.POINTER(_P), ctypes.POINTER(_P)]),
    "drt_session_close": (None, [_P]),
    "drt_selector_scratch_bytes": (ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int32]),
    "drt_selector_rows": (ctypes.c_int, [_P, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                         ctypes.c_double, _P, _P, _P, _P]),
    "drt_selector_rows_noalloc": (ctypes.c_int, [_P, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                                 ctypes.c_double, _P, _P, _P]),
    "drt_selector_gather": (ctypes.c_int, [_P, ctypes.c_int64, _P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                           ctypes.c_double, _P, _P, _P, _P]),
    "drt_selector_topp": (ctypes.c_int, [_P, ctypes.c_int64, _P, ctypes.c_int32, ctypes.c_int32, ctypes.c_double,
                                         ctypes.c_double, ctypes.c_int32, ctypes.c_double, _P, _P, _P, _P]),
    "drt_selector_sample": (ctypes.c_int, [_P, ctypes.c_int64, _P, ctypes.c_int32, ctypes.c_int32, ctypes.c_double,
                                           ctypes.c_uint64, ctypes.c_int32, _P, _P, _P, _P, _P, _P]),
    "drt_exp_nonpos": (ctypes.c_int, [_P, _P, ctypes.c_int64, _P]),
    "drt_select_choices": (ctypes.c_int, [_P, _P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_double,
                                          ctypes.c_double, _P, _P, _P]),
    "drt_quantize_q4": (ctypes.c_int, [_P, ctypes.c_int64, ctypes.c_int32, _P, _P, _P, _P]),
    "drt_linear_q4": (ctypes.c_int, [_P, _P, _P, _P, _P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                     _P]),
    "drt_quantize_q8": (ctypes.c_int, [_P, ctypes.c_int64, ctypes.c_int32, _P, _P, _P, _P]),
    "drt_linear_q8": (ctypes.c_int, [_P, _P, _P, _P, _P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                     _P]),
    "drt_linear_scratch_bytes": (ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
    "drt_linear_bf16": (ctypes.c_int, [_P, _P, _P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                       ctypes.c_int32, _P, _P]),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load the in-tree shared library and bind every entry point (raises if it is missing)."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("DIFFUSORRT_B200_LIB", LIB_PATH))
    if not path.exists():
        raise RuntimeError(f"{path} is missing; build it with `python -m diffusorrt_b200.build` "
                           "(this package has no CPU fallback)")
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int) -> None:
    if status != OK:
        msg = load().drt_last_error().decode("utf-8", "replace")
        raise DrtError(status, msg)


def i32_array(values):
    values = list(values)
    arr = (ctypes.c_int32 * max(1, len(values)))(*values)
    return arr
