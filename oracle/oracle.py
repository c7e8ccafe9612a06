"""ORACLE — test infrastructure only (never imported by the product path).

ctypes binding of ``oracle/oracle.cpp``, the C++ restatement of the reference's CPU
sampler (``src/runtime/sampling.ts:1-96`` and ``src/runtime/constraints.ts:159-173`` of
aribornstein/gemma-webgpu-engine).  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline / ``--impl reference`` legs of ``bench.py`` may import this module.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")


class OracleConfig(ctypes.Structure):
    _fields_ = [
        ("temperature", ctypes.c_double),
        ("top_p", ctypes.c_double),
        ("min_p", ctypes.c_double),
        ("typical_p", ctypes.c_double),
        ("repetition_penalty", ctypes.c_double),
        ("presence_penalty", ctypes.c_double),
        ("frequency_penalty", ctypes.c_double),
        ("top_k", ctypes.c_int32),
        ("repetition_window", ctypes.c_int32),
    ]


class OracleTrace(ctypes.Structure):
    _fields_ = [
        ("total", ctypes.c_double),
        ("max_key", ctypes.c_double),
        ("candidate_total", ctypes.c_double),
        ("uniform", ctypes.c_double),
        ("margin_top_p", ctypes.c_double),
        ("margin_draw", ctypes.c_double),
        ("margin_min_p", ctypes.c_double),
        ("margin_typical", ctypes.c_double),
        ("n_after_top_k", ctypes.c_int32),
        ("n_after_min_p", ctypes.c_int32),
        ("n_after_typical", ctypes.c_int32),
        ("n_final", ctypes.c_int32),
        ("fell_through", ctypes.c_int32),
        ("greedy", ctypes.c_int32),
    ]


def build() -> str:
    """Compile the oracle shared object (make -C oracle)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        L.oracle_seeded_init.argtypes = [ctypes.c_double]
        L.oracle_seeded_init.restype = ctypes.c_double
        L.oracle_seeded_next.argtypes = [ctypes.POINTER(ctypes.c_double)]
        L.oracle_seeded_next.restype = ctypes.c_double
        L.oracle_sample_token.argtypes = [P, ctypes.c_int64, P, ctypes.c_int64, ctypes.POINTER(OracleConfig),
                                          ctypes.c_double, P, P, P, ctypes.c_int64, ctypes.POINTER(OracleTrace)]
        L.oracle_sample_token.restype = ctypes.c_int32
        L.oracle_sample_token_seeded.argtypes = [P, ctypes.c_int64, P, ctypes.c_int64, ctypes.POINTER(OracleConfig),
                                                 ctypes.POINTER(ctypes.c_double), P, P, P, ctypes.c_int64,
                                                 ctypes.POINTER(OracleTrace)]
        L.oracle_sample_token_seeded.restype = ctypes.c_int32
        L.oracle_token_log_probability.argtypes = [P, ctypes.c_int64, ctypes.c_int64, ctypes.POINTER(ctypes.c_int32)]
        L.oracle_token_log_probability.restype = ctypes.c_double
        L.oracle_mask_constraint_logits.argtypes = [P, ctypes.c_int64, P, ctypes.c_int64, P, ctypes.c_int64, P]
        L.oracle_softcap.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_float]
        L.oracle_softcap.restype = ctypes.c_float
        L.oracle_softcap_array.argtypes = [P, P, ctypes.c_int64, ctypes.c_float, ctypes.c_float]
        L.oracle_softcap_digest.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float, ctypes.c_float, ctypes.c_int]
        L.oracle_softcap_digest.restype = ctypes.c_uint64
        L.oracle_softcap_check.argtypes = [ctypes.c_float, ctypes.c_int, ctypes.POINTER(ctypes.c_double),
                                           ctypes.POINTER(ctypes.c_uint64)]
        L.oracle_softcap_check.restype = None
        L.oracle_constraint_masks.argtypes = [ctypes.c_int32, P, P, P, P, P, ctypes.c_int64, P, P, ctypes.c_int32,
                                              P, P, P, P, ctypes.c_int64, P, ctypes.c_int64, P, ctypes.c_int64, P]
        L.oracle_constraint_masks.restype = None
        L.oracle_mask_reasoning_logits.argtypes = [P, ctypes.c_int64, P, ctypes.c_int32, ctypes.c_int64, P]
        L.oracle_mask_reasoning_logits.restype = None
        L.oracle_sample_rows.argtypes = [P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_float,
                                         P, ctypes.c_int64, P, P, ctypes.c_int64, P,
                                         P, ctypes.c_int32, P, P, P, P, ctypes.c_int, P, P, P, ctypes.c_int64]
        L.oracle_lm_head_shader_f32.argtypes = [P, P, ctypes.c_int64, ctypes.c_int, P, P, ctypes.c_int,
                                                ctypes.c_float, P, ctypes.c_int64]
        L.oracle_lm_head_shader_f32.restype = None
        L.oracle_lm_head_exact.argtypes = [P, P, ctypes.c_int64, ctypes.c_int, P, P, ctypes.c_int, ctypes.c_float,
                                           ctypes.c_float, P, ctypes.c_int64]
        L.oracle_lm_head_exact.restype = None
        _lib = L
    return _lib


def make_config(d: dict) -> OracleConfig:
    return OracleConfig(
        float(d["temperature"]), float(d["topP"]), float(d["minP"]), float(d["typicalP"]),
        float(d["repetitionPenalty"]), float(d["presencePenalty"]), float(d["frequencyPenalty"]),
        int(d["topK"]), int(d["repetitionWindow"]))


@dataclass
class OracleResult:
    token: int
    candidates: list
    probabilities: list
    trace: OracleTrace


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32).reshape(-1))


def sample_token(raw_logits, history, config: dict, uniform: float | None = None,
                 rng_state: float | None = None, cand_cap: int | None = None):
    """sampleToken restated.  Give either ``uniform`` (the random() value) or
    ``rng_state`` (a SeededRandom state, returned advanced).  Returns
    (OracleResult, new_rng_state)."""
    x = _f32(raw_logits)
    h = _i32(history if history is not None else [])
    V = x.size
    cap = V if cand_cap is None else cand_cap
    ids = np.zeros(max(cap, 1), dtype=np.int32)
    probs = np.zeros(max(cap, 1), dtype=np.float64)
    cnt = ctypes.c_int32(0)
    tr = OracleTrace()
    cfg = make_config(config)
    L = lib()
    if rng_state is not None:
        st = ctypes.c_double(rng_state)
        tok = L.oracle_sample_token_seeded(x.ctypes.data, V, h.ctypes.data, h.size, ctypes.byref(cfg),
                                           ctypes.byref(st), ids.ctypes.data, probs.ctypes.data,
                                           ctypes.byref(cnt), cap, ctypes.byref(tr))
        new_state = st.value
    else:
        u = math.nan if uniform is None else float(uniform)
        tok = L.oracle_sample_token(x.ctypes.data, V, h.ctypes.data, h.size, ctypes.byref(cfg), u,
                                    ids.ctypes.data, probs.ctypes.data, ctypes.byref(cnt), cap,
                                    ctypes.byref(tr))
        new_state = None
    n = min(cnt.value, cap)
    return OracleResult(int(tok), ids[:n].tolist(), probs[:n].tolist(), tr), new_state


def seeded_init(seed: float) -> float:
    return lib().oracle_seeded_init(float(seed))


def seeded_next(state: float):
    st = ctypes.c_double(state)
    v = lib().oracle_seeded_next(ctypes.byref(st))
    return v, st.value


def token_log_probability(raw_logits, token: int) -> float:
    x = _f32(raw_logits)
    err = ctypes.c_int32(0)
    v = lib().oracle_token_log_probability(x.ctypes.data, x.size, int(token), ctypes.byref(err))
    if err.value:
        raise ValueError(f"Token {token} is outside logits length {x.size}")
    return v


def mask_constraint_logits(raw_logits, legal, termination) -> np.ndarray:
    x = _f32(raw_logits)
    lg = _i32(legal)
    tm = _i32(termination)
    out = np.empty_like(x)
    lib().oracle_mask_constraint_logits(x.ctypes.data, x.size, lg.ctypes.data, lg.size, tm.ctypes.data,
                                        tm.size, out.ctypes.data)
    return out


def mask_reasoning_logits(raw_logits, has_bytes, allow_end: bool, end_id: int = 101) -> np.ndarray:
    """maskReasoningLogits restated (src/runtime/gemma-session.ts:1331-1345)."""
    x = _f32(raw_logits)
    hb = np.ascontiguousarray(np.asarray(has_bytes, dtype=bool).astype(np.uint8))
    assert hb.size == x.size
    out = np.empty_like(x)
    lib().oracle_mask_reasoning_logits(x.ctypes.data, x.size, hb.ctypes.data, 1 if allow_end else 0, int(end_id),
                                       out.ctypes.data)
    return out


def softcap(x, cap: float) -> np.ndarray:
    a = _f32(x)
    out = np.empty_like(a)
    inv = np.float32(1.0 / float(cap))
    lib().oracle_softcap_array(a.ctypes.data, out.ctypes.data, a.size, float(np.float32(cap)), float(inv))
    return out


def softcap_digest(lo: int, hi: int, cap: float, threads: int = 0) -> int:
    inv = np.float32(1.0 / float(cap))
    if threads <= 0:
        threads = os.cpu_count() or 1
    return int(lib().oracle_softcap_digest(lo, hi, float(np.float32(cap)), float(inv), threads))


def softcap_check(cap: float, threads: int = 0) -> tuple[float, int]:
    """(largest error in ulps against cap·tanh(x/cap), number of decreasing steps) over
    every positive float32 input."""
    if threads <= 0:
        threads = os.cpu_count() or 1
    u, d = ctypes.c_double(), ctypes.c_uint64()
    lib().oracle_softcap_check(float(np.float32(cap)), threads, ctypes.byref(u), ctypes.byref(d))
    return u.value, int(d.value)


def lm_head(packed, scales, act, act_sum, out_scale: float = 0.0, in_scale: float | None = None) -> np.ndarray:
    """Logits [rows, V] of the int2 LM head (decode-lm-head.ts): `in_scale` None restates
    the WGSL shader's f32 arithmetic; a number gives the exact computation the CUDA path
    performs (int8 activation codes when in_scale != 0, double sums when 0)."""
    packed = np.ascontiguousarray(packed, np.uint32)
    V, words = packed.shape
    sc = _f32(scales)
    a = np.ascontiguousarray(np.atleast_2d(act), np.float32)
    rows, hidden = a.shape
    assert hidden == 16 * words
    s = _f32(np.atleast_1d(act_sum))
    out = np.empty((rows, V), np.float32)
    if in_scale is None:
        lib().oracle_lm_head_shader_f32(packed.ctypes.data, sc.ctypes.data, V, hidden, a.ctypes.data, s.ctypes.data,
                                        rows, float(np.float32(out_scale)), out.ctypes.data, V)
    else:
        lib().oracle_lm_head_exact(packed.ctypes.data, sc.ctypes.data, V, hidden, a.ctypes.data, s.ctypes.data,
                                   rows, float(np.float32(in_scale)), float(np.float32(out_scale)), out.ctypes.data, V)
    return out


def constraint_masks(dfa, vocab, node, pending_len=None, pending_bytes=None, termination=(), extra=(),
                     mask_words=None):
    """Bitmask rows [states, mask_words] and dead-end flags of the constraint states
    (legalTokenIds over the token-byte trie, then selectConstrainedToken's rule).
    `dfa` is (range_offsets, range_lo, range_hi, range_target, final) and `vocab`
    (offsets, bytes), numpy arrays."""
    off, lo, hi, tgt, fin = (np.ascontiguousarray(dfa[0], np.int32), np.ascontiguousarray(dfa[1], np.uint32),
                             np.ascontiguousarray(dfa[2], np.uint32), np.ascontiguousarray(dfa[3], np.int32),
                             np.ascontiguousarray(dfa[4], np.uint8))
    toff, tb = np.ascontiguousarray(vocab[0], np.int64), np.ascontiguousarray(vocab[1], np.uint8)
    V = len(toff) - 1
    node = np.ascontiguousarray(node, np.int32)
    S = len(node)
    plen = np.zeros(S, np.uint8) if pending_len is None else np.ascontiguousarray(pending_len, np.uint8)
    pb = np.zeros(3 * S, np.uint8) if pending_bytes is None else np.ascontiguousarray(pending_bytes, np.uint8)
    term = np.ascontiguousarray(termination, np.int32)
    ext = np.ascontiguousarray(extra, np.int32)
    W = mask_words or (V + 31) // 32
    table = np.zeros((S, W), np.uint32)
    dead = np.zeros(S, np.int32)
    tb_ptr = tb.ctypes.data if tb.size else None
    lib().oracle_constraint_masks(len(fin), off.ctypes.data, lo.ctypes.data, hi.ctypes.data, tgt.ctypes.data,
                                  fin.ctypes.data, V, toff.ctypes.data, tb_ptr, S, node.ctypes.data,
                                  plen.ctypes.data, pb.ctypes.data, term.ctypes.data if term.size else None,
                                  term.size, ext.ctypes.data if ext.size else None, ext.size, table.ctypes.data, W,
                                  dead.ctypes.data)
    return table, dead


def sample_rows(logits: np.ndarray, vocab: int, softcap_value: float, history: np.ndarray | None,
                history_len: np.ndarray | None, mask_table: np.ndarray | None, mask_state: np.ndarray | None,
                configs: list, rng_state: np.ndarray | None = None, uniforms: np.ndarray | None = None,
                threads: int = 1, cand_cap: int = 0):
    """Batched restatement (rows independent, split across host threads).
    Returns (ids, traces, advanced rng_state); with cand_cap > 0 also each row's final
    candidate list as (ids [rows, cand_cap], probabilities [rows, cand_cap], counts [rows]),
    a count above cand_cap meaning a list longer than the arrays."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows = logits.shape[0]
    stride = logits.shape[1]
    hist = None if history is None else np.ascontiguousarray(history, dtype=np.int32)
    hlen = None if history_len is None else np.ascontiguousarray(history_len, dtype=np.int32)
    mt = None if mask_table is None else np.ascontiguousarray(mask_table, dtype=np.uint32)
    ms = None if mask_state is None else np.ascontiguousarray(mask_state, dtype=np.int32)
    cfgs = (OracleConfig * len(configs))(*[make_config(c) for c in configs])
    per_row = 1 if len(configs) == rows and rows > 1 else 0
    st = None if rng_state is None else np.ascontiguousarray(rng_state, dtype=np.float64).copy()
    un = None if uniforms is None else np.ascontiguousarray(uniforms, dtype=np.float64)
    ids = np.zeros(rows, dtype=np.int32)
    traces = (OracleTrace * rows)()

    def ptr(a):
        return None if a is None else a.ctypes.data

    cids = cprobs = ccount = None
    if cand_cap > 0:
        cids = np.zeros((rows, cand_cap), dtype=np.int32)
        cprobs = np.zeros((rows, cand_cap), dtype=np.float64)
        ccount = np.zeros(rows, dtype=np.int32)
    lib().oracle_sample_rows(logits.ctypes.data, rows, vocab, stride, float(softcap_value),
                             ptr(hist), 0 if hist is None else hist.shape[1], ptr(hlen),
                             ptr(mt), 0 if mt is None else mt.shape[1], ptr(ms),
                             cfgs, per_row, ptr(st), ptr(un), ids.ctypes.data, traces, int(threads),
                             ptr(cids), ptr(cprobs), ptr(ccount), int(cand_cap))
    if cand_cap > 0:
        return ids, traces, st, (cids, cprobs, ccount)
    return ids, traces, st
