"""Histogram path (topK 0 or topK > 1024) against the oracle on GPU.

Covers the cases where the crossing bins sit in unusual places: constrained rows with
penalties, topK above the candidate path's limit, min-p, topP 1 (the draw over every
finite candidate, and over the -inf group when ids are masked), -inf logits, a peaked row
whose tail falls in the deepest bin, small and unaligned vocabularies, bf16 logits, a
batch mixing both paths, and bit-identical replays.
"""
from __future__ import annotations

import importlib

import numpy as np
import pytest

import parity_util as PU

pytestmark = pytest.mark.gpu


def _p(**kw):
    p = {"temperature": 1.0, "topK": 0, "topP": 0.9, "minP": 0.0, "typicalP": 1.0, "repetitionPenalty": 1.0,
         "presencePenalty": 0.0, "frequencyPenalty": 0.0, "repetitionWindow": 0}
    p.update(kw)
    return p


def _check(oracle, sampler, x, params, *, softcap=30.0, hist=None, hlen=None, table=None, mstate=None, seed=0,
           dtype=None, label="", max_boundary=1):
    rows, V = x.shape
    u = np.random.default_rng(seed).random(rows)
    gpu = PU.run_gpu(sampler, x, params, softcap=softcap, history=hist, history_len=hlen, mask_table=table,
                     mask_state=mstate, uniforms=u, dtype=dtype)
    xo = x
    if dtype is not None:
        import torch
        xo = torch.from_numpy(x).to(dtype).float().numpy()
    ids, margins, cands, _ = PU.oracle_rows(oracle, xo, V, softcap, params, history=hist, history_len=hlen,
                                            mask_table=table, mask_state=mstate, uniforms=u)
    assert PU.compare(gpu, ids, margins, cands, label=label) <= max_boundary
    large = importlib.import_module("gemma-webgpu-engine_b200")._lib.FLAG_LARGE_PATH
    return gpu, large


def _mask(rng, V, dens):
    allowed = rng.random((len(dens), V)) < np.array(dens)[:, None]
    allowed[:, 7] = True
    bits = allowed.reshape(len(dens), V // 32, 32).astype(np.uint64) << np.arange(32, dtype=np.uint64)
    return bits.sum(axis=-1).astype(np.uint32)


def test_constrained_with_penalties(oracle, sampler):
    rng = np.random.default_rng(1)
    V, rows, H = 65536, 12, 300
    x = (rng.standard_normal((rows, V)) * 2.0).astype(np.float32)
    table = _mask(rng, V, [0.01, 0.05, 0.3])
    mstate = np.array([(i % 4) - 1 for i in range(rows)], dtype=np.int32)
    hist = rng.integers(0, V, (rows, H)).astype(np.int32)
    hist[::2, :50] = np.argsort(-x[::2], axis=1)[:, :50]  # penalise the top of some rows
    hlen = np.full(rows, H, dtype=np.int32)
    p = _p(temperature=0.9, topP=0.95, repetitionPenalty=1.3, presencePenalty=0.4, frequencyPenalty=0.2,
           repetitionWindow=H)
    gpu, large = _check(oracle, sampler, x, [p], hist=hist, hlen=hlen, table=table, mstate=mstate, label="masked")
    assert (gpu.flags & large).all()


@pytest.mark.parametrize("k", [1500, 5000], ids=["k1500", "k5000"])
def test_topk_above_candidate_limit(oracle, sampler, k):
    rng = np.random.default_rng(k)
    x = (rng.standard_normal((6, 32768)) * 1.5).astype(np.float32)
    _check(oracle, sampler, x, [_p(topK=k, topP=1.0, temperature=1.3)], label=f"k{k}")
    _check(oracle, sampler, x, [_p(topK=k, topP=0.99, temperature=2.0)], label=f"k{k}-p", seed=3)


@pytest.mark.parametrize("minp", [0.001, 0.05, 0.5])
def test_min_p(oracle, sampler, minp):
    rng = np.random.default_rng(int(minp * 1e4))
    x = (rng.standard_normal((8, 65536)) * 2.5).astype(np.float32)
    _check(oracle, sampler, x, [_p(minP=minp, topP=1.0, temperature=0.8)], label=f"minp{minp}")
    _check(oracle, sampler, x, [_p(minP=minp, topP=0.8, temperature=1.1)], label=f"minp{minp}-p", seed=5)


def test_top_p_one_draws_over_every_candidate(oracle, sampler):
    """topP 1: L is every candidate; with masked ids L runs into the -inf group."""
    rng = np.random.default_rng(9)
    V, rows = 32768, 8
    x = (rng.standard_normal((rows, V)) * 0.5).astype(np.float32)
    _check(oracle, sampler, x, [_p(topP=1.0, temperature=1.0)], label="all-finite")
    table = _mask(rng, V, [0.5])
    mstate = np.array([0, -1] * (rows // 2), dtype=np.int32)
    _check(oracle, sampler, x, [_p(topP=1.0, temperature=1.0)], table=table, mstate=mstate, label="masked-all", seed=2)


def test_negative_infinity_logits(oracle, sampler):
    rng = np.random.default_rng(11)
    V, rows = 32768, 6
    x = (rng.standard_normal((rows, V)) * 2.0).astype(np.float32)
    x[:, rng.choice(V, V // 3, replace=False)] = -np.inf
    _check(oracle, sampler, x, [_p(topP=0.9)], softcap=0.0, label="neginf-p")
    _check(oracle, sampler, x, [_p(topP=1.0)], softcap=0.0, label="neginf-all", seed=4)


def test_peaked_row_with_deep_tail(oracle, sampler):
    """A few large logits and a bulk 40+ keys below: the bulk lands in the deepest bin."""
    rng = np.random.default_rng(13)
    V, rows = 65536, 6
    x = (rng.standard_normal((rows, V)) * 1.0).astype(np.float32)
    for r in range(rows):
        x[r, rng.choice(V, 5, replace=False)] = 25.0 - np.arange(5, dtype=np.float32) * 0.7
    _check(oracle, sampler, x, [_p(topP=0.95, temperature=0.5)], label="peaked")
    _check(oracle, sampler, x, [_p(topP=0.999999, temperature=0.5)], label="peaked-tail", seed=6)


def test_small_and_unaligned_vocabularies(oracle, sampler):
    rng = np.random.default_rng(17)
    for V in (1100, 2000, 4099, 50001):
        x = (rng.standard_normal((4, V)) * 2.0).astype(np.float32)
        _check(oracle, sampler, x, [_p(topP=0.93, temperature=0.9)], label=f"V{V}", seed=V)


def test_bf16_logits(oracle, sampler):
    import torch
    rng = np.random.default_rng(19)
    x = (rng.standard_normal((8, 65536)) * 2.0).astype(np.float32)
    _check(oracle, sampler, x, [_p(topP=0.9, temperature=1.0)], dtype=torch.bfloat16, label="bf16")


def test_mixed_batch_both_paths(oracle, sampler):
    rng = np.random.default_rng(23)
    V, rows = 65536, 8
    x = (rng.standard_normal((rows, V)) * 2.0).astype(np.float32)
    ps = [_p(topK=0 if r % 2 else 40, topP=0.9, temperature=0.8 + 0.1 * r) for r in range(rows)]
    gpu, large = _check(oracle, sampler, x, ps, label="mixed")
    assert [(f & large) != 0 for f in gpu.flags] == [r % 2 == 1 for r in range(rows)]


def test_c2_replay_is_bit_identical(sampler):
    import torch
    W = importlib.import_module("gemma-webgpu-engine_b200.workloads")
    wl = W.make("C2", device="cuda", rows=16)
    outs = []
    for _ in range(2):
        rng = wl.rng_state("cuda")
        r = sampler.sample(wl.logits, wl.params, softcap=wl.softcap, history=wl.history, history_len=wl.history_len,
                           rng_state=rng, logprob=True, candidates=256)
        torch.cuda.synchronize()
        outs.append([t.cpu().numpy().tobytes() for t in (r.ids, r.flags, r.logprob, r.cand_ids, r.cand_probs, rng)])
    assert outs[0] == outs[1]


def _typical_rows(gpu, large):
    assert (gpu.flags & large).all(), "rows left the histogram path"


@pytest.mark.parametrize("case", [
    dict(typicalP=0.9, topP=1.0, temperature=1.0),
    dict(typicalP=0.5, topP=0.9, temperature=1.0),
    dict(typicalP=0.2, topP=1.0, temperature=0.7),
    dict(typicalP=0.95, topP=0.8, minP=0.01, temperature=1.1),
    dict(typicalP=0.99, topP=1.0, minP=0.3, temperature=1.0),
    dict(typicalP=0.9, topP=0.95, topK=5000, temperature=1.3),
    dict(typicalP=0.7, topP=1.0, temperature=3.0),
], ids=["t0.9", "t0.5-p0.9", "t0.2-cold", "t0.95-minp", "t0.99-minp-all", "t0.9-k5000", "t0.7-flat"])
def test_typical_p(oracle, sampler, case):
    """typical-p over the whole vocabulary: the surprise centre from the binned first
    moments, the two ends of the typical run from the annulus bins."""
    rng = np.random.default_rng(int(case["typicalP"] * 100) + int(case["temperature"] * 10))
    V, rows = 65536, 8
    x = (rng.standard_normal((rows, V)) * 2.0).astype(np.float32)
    x[:, :64] += rng.random((rows, 64)).astype(np.float32) * 8.0  # a head above the bulk
    gpu, large = _check(oracle, sampler, x, [_p(**case)], label=f"typical-{case}", seed=7)
    _typical_rows(gpu, large)


def test_typical_p_masked_and_penalised(oracle, sampler):
    """Masked ids are -inf candidates: the reference's entropy is NaN and the typical cut
    becomes a running-sum cut; with min-p (no -inf candidate) the annulus cut runs over
    penalised entries."""
    rng = np.random.default_rng(29)
    V, rows, H = 65536, 8, 200
    x = (rng.standard_normal((rows, V)) * 2.0).astype(np.float32)
    table = _mask(rng, V, [0.2, 0.6])
    mstate = np.array([r % 3 - 1 for r in range(rows)], dtype=np.int32)
    hist = rng.integers(0, V, (rows, H)).astype(np.int32)
    hist[:, :30] = np.argsort(-x, axis=1)[:, :30]
    hlen = np.full(rows, H, dtype=np.int32)
    for i, case in enumerate([dict(typicalP=0.8, topP=0.95), dict(typicalP=0.6, topP=0.7),
                              dict(typicalP=0.9, topP=1.0, minP=0.001)]):
        p = _p(temperature=0.9, repetitionPenalty=1.3, presencePenalty=0.3, frequencyPenalty=0.1,
               repetitionWindow=H, **case)
        gpu, large = _check(oracle, sampler, x, [p], hist=hist, hlen=hlen, table=table, mstate=mstate,
                            label=f"typical-masked{i}", seed=11 + i)
        _typical_rows(gpu, large)


def test_typical_p_bf16_full_vocabulary(oracle, sampler):
    import torch
    rng = np.random.default_rng(31)
    x = (rng.standard_normal((6, 262144)) * 2.5).astype(np.float32)
    gpu, large = _check(oracle, sampler, x, [_p(typicalP=0.9, topP=0.95, temperature=1.0)], dtype=torch.bfloat16,
                        label="typical-bf16")
    _typical_rows(gpu, large)
