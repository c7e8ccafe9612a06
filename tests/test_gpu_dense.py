"""The dense streaming kernel (unconstrained rows, csrc/gs_dense.cu) against the oracle.

Batches without a constraint table and without a requested log-probability take this
kernel.  Its per-element fast path leaves three things to a per-element fix-up of the
sub-tile they fall in: penalised ids (dead), values at or beyond the soft cap, and
non-finite values.  The cases below put each of those in front of the candidate test,
the running sum's reference and the greedy argmax, at both dtypes and with and without
the soft cap, and compare every row with the oracle (candidate ids and order bit-exact,
probabilities within 1e-6 relative, ids identical unless a decision is within 1e-6 of
its boundary)."""
from __future__ import annotations

import importlib

import numpy as np
import pytest

import parity_util as PU

pytestmark = pytest.mark.gpu

W = importlib.import_module("gemma-webgpu-engine_b200.workloads")


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_c4_unmasked_4096_rows(pkg, oracle, sampler, dtype):
    """C4's rows without the constraint mask (penalty history kept), as benched."""
    import torch
    td = torch.bfloat16 if dtype == "bf16" else None
    wl = W.make("C4", device="cuda", rows=4096, dtype=td)
    x = wl.logits.float().cpu().numpy()
    hist, hlen = wl.history.cpu().numpy(), wl.history_len.cpu().numpy()
    rng = wl.rng_state("cpu").numpy()
    ps = [dict(wl.params[0], repetitionWindow=hist.shape[1])]
    gpu = PU.run_gpu(sampler, x, ps, softcap=wl.softcap, history=hist, history_len=hlen, rng_state=rng,
                     cand_cap=64, dtype=td, logprob=False)
    ids, margins, cands, st = PU.oracle_rows_batched(oracle, x, wl.vocab, wl.softcap, ps, history=hist,
                                                     history_len=hlen, rng_state=rng, cand_cap=64)
    assert PU.compare(gpu, ids, margins, cands, rng_after=st, label=f"c4-unmasked-{dtype}") <= 40


def _rows(rng, rows, V, scale):
    x = (rng.standard_normal((rows, V)) * scale).astype(np.float32)
    x[1, 1000:1040] = 9.5            # exact ties among the best values
    x[2, ::7] += 40.0                # many values past the soft cap (per-element path)
    x[3, 5] = 55.0                   # one value past the cap, the row's best
    x[4, :] = x[4, :] * 0.01         # a flat row
    x[5, 4096:8192] = 12.0           # a block of ties spanning tiles and units
    return x


@pytest.mark.parametrize("softcap", [30.0, 0.0], ids=["cap30", "nocap"])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_fixup_paths(pkg, oracle, sampler, softcap, dtype):
    """Per-row params (greedy, topK 1/7/50/112, min-p, typical-p), histories that are
    empty, spread with repeats, concentrated in one unit beyond its sorted-list size, or
    made of the row's best ids; values past the cap, ties and flat rows."""
    import torch
    rng = np.random.default_rng(11 + (softcap == 0) + 2 * (dtype == "bf16"))
    V, rows, H = 65536, 16, 600
    x = _rows(rng, rows, V, 2.5)
    if dtype == "bf16":
        x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    hist = np.zeros((rows, H), np.int32)
    hlen = np.zeros(rows, np.int32)
    for r in range(rows):
        kind = r % 4
        if kind == 1:
            h = rng.integers(0, V, H)                              # spread, repeats
        elif kind == 2:
            h = rng.choice(4096, H, replace=False)                 # > 256 ids in one unit
        elif kind == 3:
            h = np.argsort(-x[r])[:200]                            # the row's best ids
        else:
            h = np.zeros(0, np.int64)
        hist[r, :len(h)] = h
        hlen[r] = len(h)
    ps = []
    for r in range(rows):
        ps.append({"temperature": [0.0, 0.7, 1.0, 1.6][r % 4], "topK": [1, 7, 50, 112][(r // 4) % 4],
                   "topP": [0.95, 1.0, 0.6][r % 3], "minP": [0.0, 0.02][(r // 2) % 2],
                   "typicalP": [1.0, 0.9][(r // 8) % 2], "repetitionPenalty": 1.2, "presencePenalty": 0.4,
                   "frequencyPenalty": 0.2, "repetitionWindow": H})
    u = rng.random(rows)
    td = torch.bfloat16 if dtype == "bf16" else None
    gpu = PU.run_gpu(sampler, x, ps, softcap=softcap, history=hist, history_len=hlen, uniforms=u, cand_cap=128,
                     dtype=td, logprob=False)
    ids, margins, cands, _ = PU.oracle_rows_batched(oracle, x, V, softcap, ps, history=hist, history_len=hlen,
                                                    uniforms=u, cand_cap=128)
    assert PU.compare(gpu, ids, margins, cands, label=f"dense-{dtype}-{softcap}") <= 2


def test_partial_last_tile_and_small_batches(pkg, oracle, sampler):
    """A vocabulary that ends inside a tile (the last tile read element by element), at
    one row (units spread one warp per SM) and at 300 rows (full CTAs)."""
    rng = np.random.default_rng(5)
    V = 66048  # 129 tiles of 512 ids, 16-byte aligned rows
    for rows in (1, 300):
        x = (rng.standard_normal((rows, V)) * 2.0).astype(np.float32)
        x[:, V - 3] = 15.0  # the best id sits in the partial tile
        h = rng.integers(V - 400, V, (rows, 64)).astype(np.int32)
        hl = np.full(rows, 64, np.int32)
        p = {"temperature": 0.8, "topK": 40, "topP": 0.95, "minP": 0.0, "typicalP": 1.0, "repetitionPenalty": 1.1,
             "presencePenalty": 0.5, "frequencyPenalty": 0.3, "repetitionWindow": 64}
        u = rng.random(rows)
        gpu = PU.run_gpu(sampler, x, [p], softcap=30.0, history=h, history_len=hl, uniforms=u, cand_cap=64,
                         logprob=False)
        ids, margins, cands, _ = PU.oracle_rows_batched(oracle, x, V, 30.0, [p], history=h, history_len=hl,
                                                        uniforms=u, cand_cap=64)
        assert PU.compare(gpu, ids, margins, cands, label=f"partial-{rows}") <= max(1, rows // 100)


def test_nonfinite_rows_flagged(pkg, sampler):
    """NaN (any soft cap) and +inf without a soft cap flag their row; -inf without a soft
    cap is an ordinary value (probability 0); neighbours are unaffected."""
    import torch
    L = pkg._lib
    V = 32768
    x = torch.randn((4, V), device="cuda") * 2
    x[0, 12345] = float("nan")
    x[1, 777] = float("inf")
    x[2, :100] = float("-inf")
    p = {"temperature": 1.0, "topK": 20, "topP": 0.9, "minP": 0, "typicalP": 1, "repetitionPenalty": 1,
         "presencePenalty": 0, "frequencyPenalty": 0, "repetitionWindow": 0}
    u = torch.full((4,), 0.5, dtype=torch.float64, device="cuda")
    r = sampler.sample(x, p, softcap=0.0, uniforms=u)
    f = r.flags.cpu().numpy().view(np.uint32)
    assert f[0] & L.FLAG_ERR_NONFINITE and f[1] & L.FLAG_ERR_NONFINITE
    assert not (f[2] & L.FLAG_ERRORS) and not (f[3] & L.FLAG_ERRORS)
    r = sampler.sample(x, p, softcap=30.0, uniforms=u)
    f = r.flags.cpu().numpy().view(np.uint32)
    assert f[0] & L.FLAG_ERR_NONFINITE
    assert not (f[1] & L.FLAG_ERRORS) and not (f[2] & L.FLAG_ERRORS)  # capped to 30 / -30
