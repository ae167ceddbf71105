"""ctypes binding of ``libspecb200.so`` (declared in include/spec_b200.h).

This is the Python side of the C ABI.  It loads the in-tree shared library
and raises if it is missing: there is no CPU fallback anywhere in the
product path.  Status codes map onto the reference's error variants
(crates/speculate/src/error.rs:10-51).
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libspecb200.so")

SPEC_OK = 0
SPEC_ERR_INVALID = 1
SPEC_ERR_CACHE_ROLLBACK = 2
SPEC_ERR_UNSUPPORTED = 3
SPEC_ERR_IO = 4
SPEC_ERR_CUDA = 5
SPEC_ERR_OOM = 6
SPEC_ERR_TIMEOUT = 7
MAX_ROWS = 64


class SpecError(RuntimeError):
    """Base error; `code` is the C status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class SamplingError(SpecError):
    """Error::Sampling (bad argument / protocol misuse)."""


class CacheRollbackError(SpecError):
    """Error::CacheRollback."""


class UnsupportedMethodError(SpecError):
    """Error::UnsupportedMethod."""


class IoError(SpecError):
    """Error::Io (GGUF open / parse)."""


class DeviceError(SpecError):
    """Error::Other / Error::Candle: a CUDA failure, out of memory or a device timeout."""


_ERRS = {
    SPEC_ERR_INVALID: SamplingError,
    SPEC_ERR_CACHE_ROLLBACK: CacheRollbackError,
    SPEC_ERR_UNSUPPORTED: UnsupportedMethodError,
    SPEC_ERR_IO: IoError,
    SPEC_ERR_CUDA: DeviceError,
    SPEC_ERR_OOM: DeviceError,
    SPEC_ERR_TIMEOUT: DeviceError,
}

c_int_p = ctypes.POINTER(ctypes.c_int)
c_u32_p = ctypes.POINTER(ctypes.c_uint32)
c_i32_p = ctypes.POINTER(ctypes.c_int32)
c_f32_p = ctypes.POINTER(ctypes.c_float)


class EagleWeights(ctypes.Structure):
    """spec_eagle_weights (include/spec_b200.h)."""

    _fields_ = [(n, ctypes.c_void_p) for n in ("fc", "q", "k", "v", "o", "gate", "up", "down", "post_norm")] + [
        ("rope_theta", ctypes.c_float)]


class MedusaWeights(ctypes.Structure):
    """spec_medusa_weights (include/spec_b200.h)."""

    _fields_ = [("n_heads", ctypes.c_int), ("residual_layers", ctypes.c_int), ("res_w", ctypes.c_void_p),
                ("res_b", ctypes.c_void_p), ("out_w", ctypes.c_void_p)]


class LoadOpts(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("max_ctx", ctypes.c_int), ("use_graphs", ctypes.c_int),
                ("tp_rank", ctypes.c_int), ("tp_size", ctypes.c_int), ("reserved", ctypes.c_int * 3)]


class ModelDesc(ctypes.Structure):
    _fields_ = [("arch", ctypes.c_int), ("n_layers", ctypes.c_int), ("hidden", ctypes.c_int),
                ("n_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int), ("ffn", ctypes.c_int),
                ("vocab", ctypes.c_int), ("rope_theta", ctypes.c_float), ("eps", ctypes.c_float),
                ("quant_mix", ctypes.c_int), ("rope_half", ctypes.c_int), ("damp_from_layer", ctypes.c_int),
                ("damp_e4", ctypes.c_int), ("reserved", ctypes.c_int * 4)]


# (name, restype, argtypes) of every function declared in include/spec_b200.h
SIGNATURES = [
    ("spec_load_gguf", ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(LoadOpts), ctypes.POINTER(ctypes.c_void_p)]),
    ("spec_create_synthetic", ctypes.c_int,
     [ctypes.POINTER(ModelDesc), ctypes.c_uint64, ctypes.POINTER(LoadOpts), ctypes.POINTER(ctypes.c_void_p)]),
    ("spec_synthetic_seed", ctypes.c_uint64, [ctypes.c_uint64, ctypes.c_uint64]),
    ("spec_synthetic_tensor", ctypes.c_int,
     [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.c_float, ctypes.c_void_p,
      ctypes.c_int64]),
    ("spec_synthetic_vector", ctypes.c_int,
     [ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.c_float, ctypes.c_float, c_f32_p]),
    ("spec_free", None, [ctypes.c_void_p]),
    ("spec_last_error", ctypes.c_char_p, [ctypes.c_void_p]),
    ("spec_vocab_size", ctypes.c_int, [ctypes.c_void_p]),
    ("spec_hidden_size", ctypes.c_int, [ctypes.c_void_p]),
    ("spec_num_layers", ctypes.c_int, [ctypes.c_void_p]),
    ("spec_history_len", ctypes.c_int, [ctypes.c_void_p]),
    ("spec_history", ctypes.c_int, [ctypes.c_void_p, c_u32_p, ctypes.c_int]),
    ("spec_kv_len", ctypes.c_int, [ctypes.c_void_p]),
    ("spec_max_ctx", ctypes.c_int, [ctypes.c_void_p]),
    ("spec_reset", ctypes.c_int, [ctypes.c_void_p]),
    ("spec_observe", ctypes.c_int, [ctypes.c_void_p, c_u32_p, ctypes.c_int]),
    ("spec_next_logits", ctypes.c_int, [ctypes.c_void_p, c_f32_p]),
    ("spec_batched_logits", ctypes.c_int, [ctypes.c_void_p, c_u32_p, ctypes.c_int, c_f32_p]),
    ("spec_rollback_to", ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    ("spec_tree_logits", ctypes.c_int, [ctypes.c_void_p, c_u32_p, c_i32_p, ctypes.c_int, c_f32_p]),
    ("spec_tree_logits_keep_kv", ctypes.c_int, [ctypes.c_void_p, c_u32_p, c_i32_p, ctypes.c_int, c_f32_p, c_f32_p]),
    ("spec_commit_tree_path", ctypes.c_int,
     [ctypes.c_void_p, c_u32_p, c_i32_p, ctypes.c_int, c_i32_p, ctypes.c_int]),
    ("spec_last_hidden_state", ctypes.c_int, [ctypes.c_void_p, c_f32_p]),
    ("spec_observe_returning_last_hidden", ctypes.c_int, [ctypes.c_void_p, c_u32_p, ctypes.c_int, c_f32_p]),
    ("spec_apply_lm_head", ctypes.c_int, [ctypes.c_void_p, c_f32_p, ctypes.c_int, c_f32_p]),
    ("spec_eagle_attach", ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    ("spec_eagle_attach_synthetic", ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint64]),
    ("spec_eagle_draft", ctypes.c_int,
     [ctypes.c_void_p, c_f32_p, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_int,
      ctypes.POINTER(ctypes.c_int32), c_f32_p]),
    ("spec_eagle_build_tree", ctypes.c_int,
     [ctypes.c_uint32, c_i32_p, c_f32_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, c_u32_p, c_i32_p, ctypes.c_int,
      c_int_p]),
    ("spec_eagle_round", ctypes.c_int,
     [ctypes.c_void_p, c_f32_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, c_u32_p, ctypes.c_int,
      c_u32_p, c_int_p, c_f32_p, c_int_p]),
    ("spec_medusa_attach", ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    ("spec_medusa_attach_synthetic", ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_uint64]),
    ("spec_medusa_topk", ctypes.c_int,
     [ctypes.c_void_p, c_f32_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int32), c_f32_p]),
    ("spec_medusa_num_heads", ctypes.c_int, [ctypes.c_void_p]),
    ("spec_medusa_round", ctypes.c_int,
     [ctypes.c_void_p, c_f32_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int,
      c_u32_p, c_int_p, c_f32_p]),
    ("spec_sd_greedy_round", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_int)]),
    ("spec_apply_lm_head_topk", ctypes.c_int,
     [ctypes.c_void_p, c_f32_p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int32), c_f32_p]),
    ("spec_embed_tokens", ctypes.c_int, [ctypes.c_void_p, c_u32_p, ctypes.c_int, c_f32_p]),
    ("spec_last_hidden_states_multi", ctypes.c_int, [ctypes.c_void_p, c_i32_p, ctypes.c_int, c_f32_p, c_f32_p]),
    ("spec_verify_greedy", ctypes.c_int, [ctypes.c_void_p, c_u32_p, ctypes.c_int, c_int_p, c_u32_p, c_i32_p]),
    ("spec_verify_rejection", ctypes.c_int,
     [ctypes.c_void_p, c_u32_p, ctypes.c_int, c_f32_p, ctypes.c_float, c_f32_p, ctypes.c_int, ctypes.c_int, c_u32_p,
      c_int_p, c_int_p]),
    ("spec_rng_create", ctypes.c_int, [ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)]),
    ("spec_rng_free", None, [ctypes.c_void_p]),
    ("spec_rng_next_f32", ctypes.c_int, [ctypes.c_void_p, c_f32_p, ctypes.c_int]),
    ("spec_sd_sampled_round", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_int,
      ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
    ("spec_verify_tree_greedy", ctypes.c_int,
     [ctypes.c_void_p, c_u32_p, c_i32_p, ctypes.c_int, c_i32_p, c_int_p, c_u32_p]),
    ("spec_verify_tree_typical", ctypes.c_int,
     [ctypes.c_void_p, c_u32_p, c_i32_p, ctypes.c_int, ctypes.c_float, ctypes.c_float, c_i32_p, c_int_p, c_u32_p]),
    ("spec_last_forward_ms", ctypes.c_float, [ctypes.c_void_p]),
    ("spec_kernels_per_forward", ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    ("spec_cuda_stream", ctypes.c_void_p, [ctypes.c_void_p]),
    ("spec_profile_forward", ctypes.c_int,
     [ctypes.c_void_p, c_u32_p, ctypes.c_int, c_f32_p, c_int_p, ctypes.POINTER(ctypes.c_int64), ctypes.c_int]),
    ("spec_weight_bytes", ctypes.c_int64, [ctypes.c_void_p]),
    ("spec_qweight_upload", ctypes.c_int,
     [ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]),
    ("spec_qweight_free", None, [ctypes.c_void_p]),
    ("spec_qmatmul", ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    ("spec_qweight_bytes", ctypes.c_int64, [ctypes.c_void_p]),
    ("spec_qmatmul_time", ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, c_f32_p]),
    ("spec_tp_handle", ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]),
    ("spec_tp_connect", ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]),
    ("spec_tp_size", ctypes.c_int, [ctypes.c_void_p]),
    ("spec_qmatmul_noalloc", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
]

_lib: Optional[ctypes.CDLL] = None


def load() -> ctypes.CDLL:
    """Load libspecb200.so (raises FileNotFoundError if it was never built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise FileNotFoundError(
            f"{LIB_PATH} is missing: build it with `python abyo-speculate_b200/build.py` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int, handle=None) -> None:
    """Raise the error class matching status `rc` (no-op on SPEC_OK)."""
    if rc == SPEC_OK:
        return
    lib = load()
    msg = lib.spec_last_error(handle)
    text = msg.decode("utf-8", "replace") if msg else ""
    raise _ERRS.get(rc, SpecError)(rc, text)
