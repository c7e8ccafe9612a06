"""Test helpers: run the CUDA path and the CPU oracle on the same inputs and compare.

The parity bar: filtered candidate ids and their order bit-exact;
probabilities within 1e-6 relative; sampled ids identical except decisions within 1e-6
of a boundary, which are counted.  A row counts as a boundary case when the GPU flags it
(GS_FLAG_BOUNDARY_*) or the oracle's own decision margin is below 1e-6.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np

PROB_RTOL = 1e-6
BOUNDARY = 1e-6


@dataclass
class GpuOut:
    ids: np.ndarray
    flags: np.ndarray
    rng_after: np.ndarray
    cand_ids: np.ndarray
    cand_probs: np.ndarray
    cand_count: np.ndarray
    logprob: np.ndarray


def run_gpu(sampler, logits_np, params, *, softcap=0.0, history=None, history_len=None, mask_table=None,
            mask_state=None, rng_state=None, uniforms=None, cand_cap=2048, dtype=None, logprob=True,
            history_count=None):
    import torch
    dev = torch.device("cuda", 0)
    x = torch.from_numpy(np.ascontiguousarray(logits_np)).to(dev)
    if dtype is not None:
        x = x.to(dtype)
    t = lambda a, dt: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(dt)  # noqa: E731
    rng = t(rng_state, torch.float64)
    res = sampler.sample(x, params, softcap=softcap, history=t(history, torch.int32),
                         history_len=t(history_len, torch.int32),
                         mask_table=t(None if mask_table is None else mask_table.view(np.int32), torch.int32),
                         mask_state=t(mask_state, torch.int32), rng_state=rng, uniforms=t(uniforms, torch.float64),
                         logprob=logprob, candidates=cand_cap, history_count=t(history_count, torch.int32))
    torch.cuda.synchronize()
    return GpuOut(
        ids=res.ids.cpu().numpy(), flags=res.flags.cpu().numpy().view(np.uint32),
        rng_after=None if rng is None else rng.cpu().numpy(),
        cand_ids=res.cand_ids.cpu().numpy(), cand_probs=res.cand_probs.cpu().numpy(),
        cand_count=res.cand_count.cpu().numpy(), logprob=None if res.logprob is None else res.logprob.cpu().numpy())


def oracle_rows(O, logits_np, vocab, softcap, params, *, history=None, history_len=None, mask_table=None,
                mask_state=None, rng_state=None, uniforms=None, cand_cap=2048, candidates=True):
    """Oracle outputs per row: ids, margins, candidate lists, advanced states."""
    rows = logits_np.shape[0]
    ps = params if len(params) == rows else [params[0]] * rows
    ids, traces, st = O.sample_rows(logits_np, vocab, softcap, history, history_len, mask_table, mask_state, ps,
                                    rng_state=rng_state, uniforms=uniforms, threads=os.cpu_count() or 1)
    cands = []
    if candidates:
        for r in range(rows):
            row = O.softcap(logits_np[r, :vocab], softcap) if softcap else logits_np[r, :vocab].astype(np.float32)
            if mask_table is not None and mask_state[r] >= 0:
                m = mask_table[mask_state[r]]
                idx = np.arange(vocab)
                bits = (m[idx >> 5] >> (idx & 31).astype(np.uint32)) & 1
                row = np.where(bits.astype(bool), row, -np.inf).astype(np.float32)
            h = history[r, :history_len[r]] if history is not None else []
            p = dict(ps[r], repetitionWindow=len(h))
            if uniforms is not None:
                res, _ = O.sample_token(row, h, p, uniform=uniforms[r], cand_cap=cand_cap)
            else:
                res, _ = O.sample_token(row, h, p, rng_state=rng_state[r], cand_cap=cand_cap)
            assert res.token == ids[r]
            cands.append((res.candidates, res.probabilities, res.trace.n_final))
    margins = np.array([min(t.margin_top_p, t.margin_draw, t.margin_min_p, t.margin_typical) for t in traces])
    return ids, margins, cands, st


def oracle_rows_batched(O, logits_np, vocab, softcap, params, *, history=None, history_len=None, mask_table=None,
                        mask_state=None, rng_state=None, uniforms=None, cand_cap=64):
    """oracle_rows over all host threads in one call (the batched restatement also writes
    each row's candidate list): the same outputs at full batch sizes in seconds."""
    rows = logits_np.shape[0]
    ps = params if len(params) == rows else [params[0]] * rows
    ids, traces, st, (cid, cpr, cnt) = O.sample_rows(
        logits_np, vocab, softcap, history, history_len, mask_table, mask_state, ps, rng_state=rng_state,
        uniforms=uniforms, threads=os.cpu_count() or 1, cand_cap=cand_cap)
    cands = []
    for r in range(rows):
        n = int(cnt[r])
        m = min(n, cand_cap)
        cands.append((cid[r, :m].tolist(), cpr[r, :m].tolist(), n))
    margins = np.array([min(t.margin_top_p, t.margin_draw, t.margin_min_p, t.margin_typical) for t in traces])
    return ids, margins, cands, st


def compare(gpu: GpuOut, ids, margins, cands, *, rng_after=None, label=""):
    """Asserts the parity bar; returns the number of boundary rows that differ."""
    from importlib import import_module
    L = import_module("gemma-webgpu-engine_b200")._lib
    rows = len(ids)
    boundary_diffs = 0
    for r in range(rows):
        flagged = bool(gpu.flags[r] & L.FLAG_BOUNDARY) or margins[r] < BOUNDARY
        assert not (gpu.flags[r] & L.FLAG_ERRORS), f"{label} row {r}: error flags {gpu.flags[r]:#x}"
        if gpu.ids[r] != ids[r]:
            assert flagged, f"{label} row {r}: gpu {gpu.ids[r]} oracle {ids[r]} (margin {margins[r]:.3g})"
            boundary_diffs += 1
            continue
        if cands and not flagged:
            cid, cpr = cands[r][0], cands[r][1]
            total = cands[r][2] if len(cands[r]) > 2 else len(cid)
            n = int(gpu.cand_count[r])
            assert n == total, f"{label} row {r}: {n} candidates vs {total}"
            m = min(n, gpu.cand_ids.shape[1], len(cid))
            assert gpu.cand_ids[r, :m].tolist() == list(cid[:m]), f"{label} row {r}: candidate order"
            ref = np.asarray(cpr[:m])
            got = gpu.cand_probs[r, :m]
            tol = PROB_RTOL * np.abs(ref) + 1e-300
            bad = np.abs(got - ref) > tol
            assert not bad.any(), f"{label} row {r}: prob {got[bad][:3]} vs {ref[bad][:3]}"
    if rng_after is not None and gpu.rng_after is not None:
        assert gpu.rng_after.tolist() == list(rng_after), f"{label}: rng states"
    return boundary_diffs
