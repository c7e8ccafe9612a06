"""ctypes binding of libgsampler.so (the C ABI in include/gsampler.h).

The shared object is built in-tree (``make -C gemma-webgpu-engine_b200``).  There is no
fallback: if it is missing or cannot be loaded, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgsampler.so")

GS_OK = 0
GS_EINVAL = 1
GS_EDEADEND = 2
GS_ECUDA = 3
GS_ENCCL = 4
GS_ETIMEOUT = 5
GS_ENOMEM = 6
GS_EUNSUPPORTED = 7
GS_EEMPTY = 8
GS_ENONFINITE = 9

GS_DTYPE_F32 = 0
GS_DTYPE_BF16 = 1

LM_ROUTE_AUTO = 0
LM_ROUTE_FUSED = 1
LM_ROUTE_TWO_STEP = 2

FLAG_BOUNDARY_TOP_P = 1 << 0
FLAG_BOUNDARY_DRAW = 1 << 1
FLAG_BOUNDARY_MIN_P = 1 << 2
FLAG_BOUNDARY_TYPICAL = 1 << 3
FLAG_FELL_THROUGH = 1 << 4
FLAG_GREEDY = 1 << 5
FLAG_LARGE_PATH = 1 << 6
FLAG_ERR_DEADEND = 1 << 8
FLAG_ERR_NONFINITE = 1 << 9
FLAG_ERR_INVALID = 1 << 10
FLAG_ERR_UNSUPPORTED = 1 << 11
FLAG_ERR_TIMEOUT = 1 << 12
FLAG_ERRORS = 0xFF00
FLAG_BOUNDARY = FLAG_BOUNDARY_TOP_P | FLAG_BOUNDARY_DRAW | FLAG_BOUNDARY_MIN_P | FLAG_BOUNDARY_TYPICAL

MAX_TOP_K = 1024
MAX_HISTORY = 4096

# Every symbol include/gsampler.h declares.
EXPORTS = (
    "gs_create", "gs_destroy", "gs_reserve", "gs_last_error", "gs_sample", "gs_sample_host",
    "gs_token_log_probability", "gs_mask_constraint_logits", "gs_build_mask_row", "gs_softcap",
    "gs_softcap_digest", "gs_shard_record_bytes", "gs_shard_partials", "gs_shard_merge", "gs_profile_enable",
    "gs_profile_read", "gs_sample_noalloc", "gs_constraint_create", "gs_constraint_destroy",
    "gs_constraint_last_error", "gs_constraint_build_masks", "gs_lm_head_create", "gs_lm_head_destroy",
    "gs_lm_head_last_error", "gs_lm_head_logits", "gs_lm_head_sample", "gs_lm_head_check",
    "gs_lm_head_fused_calls", "gs_build_reasoning_mask_rows", "gs_nccl_unique_id", "gs_nccl_create",
    "gs_nccl_destroy", "gs_nccl_last_error", "gs_shard_sample", "gs_lm_head_set_route",
)

NOALLOC_SCRATCH_BYTES = 8 << 20


class GsParams(ctypes.Structure):
    _fields_ = [
        ("temperature", ctypes.c_double),
        ("top_p", ctypes.c_double),
        ("min_p", ctypes.c_double),
        ("typical_p", ctypes.c_double),
        ("repetition_penalty", ctypes.c_double),
        ("presence_penalty", ctypes.c_double),
        ("frequency_penalty", ctypes.c_double),
        ("top_k", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class GsDfaDesc(ctypes.Structure):
    _fields_ = [
        ("nodes", ctypes.c_int32),
        ("range_offsets", ctypes.c_void_p),
        ("range_lo", ctypes.c_void_p),
        ("range_hi", ctypes.c_void_p),
        ("range_target", ctypes.c_void_p),
        ("final", ctypes.c_void_p),
    ]


class GsVocabBytesDesc(ctypes.Structure):
    _fields_ = [
        ("vocab", ctypes.c_int64),
        ("offsets", ctypes.c_void_p),
        ("bytes", ctypes.c_void_p),
    ]


class GsLmHeadDesc(ctypes.Structure):
    _fields_ = [
        ("vocab", ctypes.c_int64),
        ("hidden", ctypes.c_int32),
        ("packed", ctypes.c_void_p),
        ("row_scales", ctypes.c_void_p),
        ("input_scale", ctypes.c_float),
        ("output_scale", ctypes.c_float),
    ]


class GsBatch(ctypes.Structure):
    _fields_ = [
        ("logits", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("rows", ctypes.c_int32),
        ("vocab", ctypes.c_int64),
        ("row_stride", ctypes.c_int64),
        ("softcap", ctypes.c_float),
        ("params_count", ctypes.c_int32),
        ("params", ctypes.c_void_p),
        ("history", ctypes.c_void_p),
        ("history_len", ctypes.c_void_p),
        ("history_stride", ctypes.c_int64),
        ("mask_table", ctypes.c_void_p),
        ("mask_states", ctypes.c_int64),
        ("mask_words", ctypes.c_int64),
        ("mask_state", ctypes.c_void_p),
        ("rng_state", ctypes.c_void_p),
        ("uniforms", ctypes.c_void_p),
        ("history_count", ctypes.c_void_p),
    ]


class GsOutputs(ctypes.Structure):
    _fields_ = [
        ("ids", ctypes.c_void_p),
        ("logprob", ctypes.c_void_p),
        ("flags", ctypes.c_void_p),
        ("cand_ids", ctypes.c_void_p),
        ("cand_probs", ctypes.c_void_p),
        ("cand_count", ctypes.c_void_p),
        ("cand_cap", ctypes.c_int32),
    ]


def build(force: bool = False) -> str:
    """Compiles libgsampler.so for sm_100a (make, nvcc)."""
    if force or not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-s", "-j8", "-C", _HERE], check=True)
    else:
        subprocess.run(["make", "-s", "-j8", "-C", _HERE], check=True)
    return LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    """Loads libgsampler.so; raises if it is not built (there is no CPU fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"libgsampler.so is not built ({LIB_PATH}); run make -C {_HERE}")
    L = ctypes.CDLL(LIB_PATH)
    P = ctypes.c_void_p
    i32, i64, f32, u64 = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_uint64
    L.gs_create.argtypes = [ctypes.c_int, ctypes.POINTER(P)]
    L.gs_destroy.argtypes = [P]
    L.gs_reserve.argtypes = [P, i32, i64, i32, i64]
    L.gs_last_error.argtypes = [P]
    L.gs_last_error.restype = ctypes.c_char_p
    L.gs_sample.argtypes = [P, ctypes.POINTER(GsBatch), ctypes.POINTER(GsOutputs), P]
    L.gs_sample_host.argtypes = [P, ctypes.POINTER(GsBatch), ctypes.POINTER(GsOutputs), P]
    L.gs_token_log_probability.argtypes = [P, P, i32, i32, i64, i64, f32, P, P, P]
    L.gs_mask_constraint_logits.argtypes = [P, P, i64, P, i64, P, i64, P, P]
    L.gs_build_mask_row.argtypes = [P, i64, P, i64, P, i64, P, P]
    L.gs_build_reasoning_mask_rows.argtypes = [P, i64, P, i32, P, i64, P]
    L.gs_constraint_create.argtypes = [P, ctypes.POINTER(GsDfaDesc), ctypes.POINTER(GsVocabBytesDesc),
                                       ctypes.POINTER(P)]
    L.gs_constraint_destroy.argtypes = [P]
    L.gs_constraint_last_error.argtypes = [P]
    L.gs_constraint_last_error.restype = ctypes.c_char_p
    L.gs_constraint_build_masks.argtypes = [P, i32, P, P, P, P, i64, P, i64, P, i64, P, P]
    L.gs_lm_head_create.argtypes = [P, ctypes.POINTER(GsLmHeadDesc), ctypes.POINTER(P)]
    L.gs_lm_head_destroy.argtypes = [P]
    L.gs_lm_head_last_error.argtypes = [P]
    L.gs_lm_head_last_error.restype = ctypes.c_char_p
    L.gs_lm_head_logits.argtypes = [P, P, i64, P, i32, P, i64, P]
    L.gs_lm_head_check.argtypes = [P, ctypes.POINTER(i32)]
    L.gs_lm_head_fused_calls.argtypes = [P]
    L.gs_lm_head_set_route.argtypes = [P, i32]
    L.gs_lm_head_sample.argtypes = [P, P, i64, P, ctypes.POINTER(GsBatch), ctypes.POINTER(GsOutputs), P]
    L.gs_softcap.argtypes = [P, P, P, i64, f32, P]
    L.gs_softcap_digest.argtypes = [P, u64, u64, f32, ctypes.POINTER(u64)]
    L.gs_shard_record_bytes.argtypes = [ctypes.POINTER(GsParams), i32, i64, i64]
    L.gs_shard_record_bytes.restype = i64
    L.gs_shard_partials.argtypes = [P, ctypes.POINTER(GsBatch), i64, i64, i32, P, P]
    L.gs_shard_merge.argtypes = [P, ctypes.POINTER(GsBatch), i32, P, ctypes.POINTER(GsOutputs), P]
    L.gs_sample_noalloc.argtypes = [ctypes.POINTER(GsBatch), ctypes.POINTER(GsOutputs), P]
    L.gs_nccl_unique_id.argtypes = [P]
    L.gs_nccl_create.argtypes = [ctypes.c_int, P, i32, i32, i32, ctypes.POINTER(P)]
    L.gs_nccl_destroy.argtypes = [P]
    L.gs_nccl_last_error.argtypes = [P]
    L.gs_nccl_last_error.restype = ctypes.c_char_p
    L.gs_shard_sample.argtypes = [P, P, ctypes.POINTER(GsBatch), i64, i64, ctypes.POINTER(GsOutputs), i32, P]
    L.gs_profile_enable.argtypes = [P, i32]
    L.gs_profile_read.argtypes = [P, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(i64),
                                  ctypes.POINTER(ctypes.c_double), ctypes.POINTER(i64)]
    for name in EXPORTS:
        if name not in ("gs_last_error", "gs_shard_record_bytes", "gs_constraint_last_error", "gs_lm_head_last_error",
                        "gs_lm_head_fused_calls", "gs_nccl_last_error"):
            getattr(L, name).restype = ctypes.c_int
    L.gs_lm_head_fused_calls.restype = i64
    _lib = L
    return L
