"""Parity at the benchmark configurations' full sizes, on the code paths the bench times.

The bench samples C4 at 4096 rows per GPU, where the merge runs one warp per row
(finalize_warp_kernel, taken when a batch has at least five rows per SM); C2's 64 rows
run the histogram path (topK 0) and C3's 256 rows the block merge.  These tests run the
configurations at BASELINE.json's batch sizes through the C ABI and compare every row
with the CPU oracle on the same bytes: candidate ids and order bit-exact, probabilities
within 1e-6 relative, ids identical unless a decision lies within 1e-6 of its boundary
(flagged or the oracle's margin), and the advanced PRNG states exactly.
"""
from __future__ import annotations

import importlib

import numpy as np
import pytest

import parity_util as PU

pytestmark = pytest.mark.gpu

W = importlib.import_module("gemma-webgpu-engine_b200.workloads")


def _full(pkg, oracle, sampler, name, rows, dtype=None, cand_cap=64, params=None, max_boundary_frac=0.01):
    wl = W.make(name, device="cuda", rows=rows, dtype=dtype)
    x = wl.logits.float().cpu().numpy()
    hist = None if wl.history is None else wl.history.cpu().numpy()
    hlen = None if wl.history_len is None else wl.history_len.cpu().numpy()
    table = None if wl.mask_table is None else wl.mask_table.cpu().numpy().view(np.uint32)
    mstate = None if wl.mask_state is None else wl.mask_state.cpu().numpy()
    rng = wl.rng_state("cpu").numpy()
    ps = params if params is not None else wl.params
    ps = [dict(p, repetitionWindow=(hist.shape[1] if hist is not None else 0)) for p in ps]
    gpu = PU.run_gpu(sampler, x, ps, softcap=wl.softcap, history=hist, history_len=hlen, mask_table=table,
                     mask_state=mstate, rng_state=rng, cand_cap=cand_cap, dtype=dtype)
    ids, margins, cands, st = PU.oracle_rows_batched(oracle, x, wl.vocab, wl.softcap, ps, history=hist,
                                                     history_len=hlen, mask_table=table, mask_state=mstate,
                                                     rng_state=rng, cand_cap=cand_cap)
    diffs = PU.compare(gpu, ids, margins, cands, rng_after=st, label=f"{name}x{rows}")
    assert diffs <= max(1, int(rows * max_boundary_frac)), diffs
    return gpu


def test_c4_f32_4096_rows_warp_merge(pkg, oracle, sampler):
    """C4 exactly as benched: 4096 rows of float32 logits on one GPU."""
    gpu = _full(pkg, oracle, sampler, "C4", 4096)
    assert (gpu.cand_count > 0).all()


def test_c4_bf16_4096_rows_warp_merge(pkg, oracle, sampler):
    import torch
    _full(pkg, oracle, sampler, "C4", 4096, dtype=torch.bfloat16)


def test_c3_256_rows(pkg, oracle, sampler):
    _full(pkg, oracle, sampler, "C3", 256)


def test_c2_64_rows_histogram_path(pkg, oracle, sampler):
    """C2: topK disabled, topP 0.9 over the full vocabulary, 1024-id histories."""
    gpu = _full(pkg, oracle, sampler, "C2", 64, cand_cap=2048)
    assert (gpu.flags & pkg._lib.FLAG_LARGE_PATH).all()


def test_c5_8_rows(pkg, oracle, sampler):
    _full(pkg, oracle, sampler, "C5", 8, cand_cap=1024)


@pytest.mark.parametrize("temp", [10.0, 100.0], ids=["T10", "T100"])
def test_histogram_path_flat_rows(pkg, oracle, sampler, temp):
    """C2's rows at high temperature: the keys of the whole vocabulary fall within a few
    units (T 10) or a fraction of a unit (T 100) of the maximum, so the nucleus holds most
    of the vocabulary and the bins around each crossing are crowded."""
    p = W.base_params(temperature=temp, topK=0, topP=0.9, repetitionPenalty=1.1, presencePenalty=0.5,
                      frequencyPenalty=0.3)
    gpu = _full(pkg, oracle, sampler, "C2", 16, cand_cap=256, params=[p])
    assert (gpu.flags & pkg._lib.FLAG_LARGE_PATH).all()


def test_c1_256_sequential_steps(pkg, oracle, sampler):
    """C1 as specified: 256 sequential steps with fresh logits, one SeededRandom stream
    (seed 42), each sampled id appended to the history (penalties off: window 0)."""
    import torch
    st_gpu = torch.tensor([pkg.SeededRandom(42).state], dtype=torch.float64, device="cuda")
    st_ref = oracle.seeded_init(42)
    history = []
    boundary = 0
    for step in range(256):
        wl = W.make("C1", device="cuda", step=step)
        res = sampler.sample(wl.logits, wl.params, softcap=wl.softcap, rng_state=st_gpu, candidates=40)
        x = wl.logits.cpu().numpy()[0]
        ref, st_ref = oracle.sample_token(oracle.softcap(x, 30.0), history, wl.params[0], rng_state=st_ref,
                                          cand_cap=40)
        tok = int(res.ids.item())
        flagged = bool(int(res.flags.item()) & pkg._lib.FLAG_BOUNDARY) or \
            min(ref.trace.margin_top_p, ref.trace.margin_draw) < PU.BOUNDARY
        if tok != ref.token:
            assert flagged, f"step {step}: gpu {tok} oracle {ref.token}"
            boundary += 1
        elif not flagged:
            n = int(res.cand_count.item())
            assert n == len(ref.candidates)
            assert res.cand_ids[0, :n].cpu().tolist() == ref.candidates, f"step {step}"
            got = res.cand_probs[0, :n].cpu().numpy()
            assert np.allclose(got, ref.probabilities, rtol=PU.PROB_RTOL, atol=0), f"step {step}"
        history.append(ref.token)
        assert float(st_gpu.item()) == st_ref, f"step {step}: rng state"
    assert boundary <= 2


@pytest.mark.parametrize("case", [dict(typicalP=0.9, topP=1.0), dict(typicalP=0.6, topP=0.9),
                                  dict(typicalP=0.95, topP=0.95, minP=0.02)], ids=["t0.9", "t0.6-p0.9", "t0.95-minp"])
def test_c2_64_rows_typical_p(pkg, oracle, sampler, case):
    """C2's 64 rows (262144 ids, 1024-id histories, penalties) with typical-p over the full
    vocabulary: the annulus cut, the typical pre-pass and the second gather."""
    base = W.make("C2", device="cpu", rows=1).params[0]
    p = dict(base, **case)
    gpu = _full(pkg, oracle, sampler, "C2", 64, cand_cap=2048, params=[p])
    assert (gpu.flags & pkg._lib.FLAG_LARGE_PATH).all()
