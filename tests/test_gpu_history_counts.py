"""Repetition windows longer than MAX_HISTORY entries (src/runtime/decoding.ts:42-44 accepts
any non-negative window) passed as their distinct ids with counts (gs_batch.history_count),
against the oracle sampling the raw window.  The penalties depend only on each id's count
in the window (src/runtime/sampling.ts:21-30), so both forms must give the same candidates,
probabilities and ids.  Each case takes one merge path: the single-launch decode step (one
row), the block merge (24 and 64 rows), the warp merge (800 rows) and the histogram path
(topK 0)."""
from __future__ import annotations

import numpy as np
import pytest

import parity_util as PU

pytestmark = pytest.mark.gpu

WINDOW = 6000  # entries per raw window: above GS_MAX_HISTORY


def _case(pkg, rows, V, distinct, seed, topk, masked):
    g = np.random.default_rng(seed)
    x = (g.standard_normal((rows, V)) * 2.0).astype(np.float32)
    raw = np.empty((rows, WINDOW), np.int32)
    for r in range(rows):
        order = np.argsort(-x[r], kind="stable")
        pool = np.concatenate([order[:8], g.integers(0, V, distinct - 10), [-3, V + 7]]).astype(np.int32)
        raw[r] = pool[g.integers(0, len(pool), WINDOW)]  # heavy repeats; the row's best ids penalised
    raw_len = np.full(rows, WINDOW, np.int32)
    raw_len[::5] = WINDOW - 1234
    comp = [pkg.compact_history(raw[r, :raw_len[r]]) for r in range(rows)]
    width = max(len(c[0]) for c in comp)
    ids = np.zeros((rows, width), np.int32)
    cnt = np.ones((rows, width), np.int32)
    lens = np.zeros(rows, np.int32)
    for r, (i, c) in enumerate(comp):
        ids[r, :len(i)] = i
        cnt[r, :len(c)] = c
        lens[r] = len(i)
    table = state = None
    if masked:
        allowed = g.random((8, V)) < 0.3
        table = np.ascontiguousarray(np.packbits(allowed, axis=1, bitorder="little").view(np.uint32))
        state = g.integers(-1, 8, rows).astype(np.int32)
    params = [dict(temperature=[0.8, 1.0, 0.0][r % 3] if rows > 1 else 0.8, topK=topk, topP=0.95, minP=0.0,
                   typicalP=1.0, repetitionPenalty=1.2, presencePenalty=0.4, frequencyPenalty=0.05,
                   repetitionWindow=WINDOW) for r in range(rows)]
    return x, raw, raw_len, ids, cnt, lens, table, state, params


@pytest.mark.parametrize("rows,V,distinct,topk,masked", [
    (1, 262144, 300, 40, False),   # single-launch decode step (<= 512 entries)
    (1, 262144, 300, 64, True),
    (24, 262144, 2000, 50, False),  # block merge, 1024 threads
    (64, 32768, 1500, 50, True),    # block merge, 512 threads
    (800, 32768, 400, 50, False),   # warp merge (<= 512 entries)
    (8, 262144, 1000, 0, False),    # histogram path (topK 0)
])
def test_long_window_as_counts_matches_oracle(pkg, oracle, sampler, rows, V, distinct, topk, masked):
    x, raw, raw_len, ids, cnt, lens, table, state, params = _case(pkg, rows, V, distinct, rows + V + topk, topk, masked)
    assert ids.shape[1] <= pkg._lib.MAX_HISTORY < WINDOW
    rng = np.array([float(900 + r) for r in range(rows)])
    gpu = PU.run_gpu(sampler, x, params, softcap=30.0, history=ids, history_len=lens, history_count=cnt,
                     mask_table=table, mask_state=state, rng_state=rng, cand_cap=64)
    ref_ids, margins, cands, st = PU.oracle_rows(oracle, x, V, 30.0, params, history=raw, history_len=raw_len,
                                                 mask_table=table, mask_state=state, rng_state=rng, cand_cap=64)
    diffs = PU.compare(gpu, ref_ids, margins, cands, rng_after=st, label=f"counts {rows}x{V}")
    assert diffs <= max(1, rows // 100), diffs


def test_sample_token_long_window(pkg, oracle):
    # the reference-facing call with a window of 8000 entries (compacted inside)
    import torch
    g = np.random.default_rng(8)
    V = 262144
    x = (g.standard_normal(V) * 2.0).astype(np.float32)
    order = np.argsort(-x, kind="stable")
    pool = np.concatenate([order[:5], g.integers(0, V, 700)])
    history = [int(v) for v in pool[g.integers(0, len(pool), 9000)]]
    cfg = dict(temperature=0.9, topK=40, topP=0.9, minP=0.0, typicalP=1.0, repetitionPenalty=1.3,
               presencePenalty=0.2, frequencyPenalty=0.1, repetitionWindow=8000)
    tok = pkg.sample_token(torch.from_numpy(x).cuda(), history, cfg, pkg.SeededRandom(5))
    res, _ = oracle.sample_token(x, history[-8000:], cfg, rng_state=pkg.SeededRandom(5).state, cand_cap=64)
    assert tok == res.token or min(res.trace.margin_top_p, res.trace.margin_draw) < 1e-6
    host_tok = pkg.sample_token(x.tolist(), history, cfg, pkg.SeededRandom(5))
    assert host_tok == tok
