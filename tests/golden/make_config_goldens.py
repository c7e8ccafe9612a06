"""Writes tests/golden/config_goldens.npz: small seeded versions of the five benchmark
configurations plus edge cases, with the CPU oracle's outputs.

Inputs come from numpy's PCG64 generator with a fixed seed per case (make_inputs); the
file keeps the oracle's outputs and a SHA-256 of every case's input bytes, so a test
that regenerates the inputs first proves they are the bytes the outputs were made from.
Run from the repository root:
    python tests/golden/make_config_goldens.py
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import oracle as O  # noqa: E402

DEFAULT = {"temperature": 0.8, "topK": 40, "topP": 0.95, "minP": 0, "typicalP": 1, "repetitionPenalty": 1.05,
           "repetitionWindow": 64, "frequencyPenalty": 0, "presencePenalty": 0}


def cfg(**kw):
    c = dict(DEFAULT)
    c.update(kw)
    return c


def seeded_state(seed):
    return O.seeded_init(seed)


def pack_bits(allowed: np.ndarray) -> np.ndarray:
    S, V = allowed.shape
    W = (V + 31) // 32
    pad = np.zeros((S, W * 32), dtype=bool)
    pad[:, :V] = allowed
    bits = pad.reshape(S, W, 32).astype(np.uint64) << np.arange(32, dtype=np.uint64)
    return bits.sum(axis=2).astype(np.uint32)


def make_inputs(name, seed, rows, vocab, kind, params, softcap=30.0, hist_len=0, states=0, density=(0.01, 0.05),
                ties=0, neg_inf=0):
    """Seeded inputs of one case (pure numpy)."""
    rng = np.random.default_rng(seed)
    if kind == "normal":
        x = rng.standard_normal((rows, vocab)) * 2.0
    elif kind == "zipf":
        perm = rng.permutation(vocab)
        bias = np.empty(vocab)
        bias[perm] = -1.1 * np.log(np.arange(1, vocab + 1))
        x = rng.standard_normal((rows, vocab)) * 2.0 + bias[None, :]
    elif kind == "gumbel":
        u = rng.random((rows, vocab)).clip(1e-300, 1 - 1e-16)
        x = -2.0 * np.log(-np.log(u))
    elif kind == "flat":
        x = np.zeros((rows, vocab))
    else:
        raise ValueError(kind)
    x = x.astype(np.float32)
    if ties:
        for r in range(rows):
            idx = rng.choice(vocab, size=min(ties, vocab), replace=False)
            x[r, idx] = x[r].max()
    if neg_inf:
        for r in range(rows):
            idx = rng.choice(vocab, size=min(neg_inf, vocab), replace=False)
            x[r, idx] = -np.inf
    hist = rng.integers(0, vocab, size=(rows, max(hist_len, 1)), dtype=np.int64).astype(np.int32)
    hlen = np.full(rows, hist_len, dtype=np.int32)
    table = None
    mstate = None
    if states:
        dens = rng.uniform(density[0], density[1], size=states)
        allowed = rng.random((states, vocab)) < dens[:, None]
        allowed[np.arange(states), rng.integers(0, vocab, size=states)] = True
        table = pack_bits(allowed)
        mstate = rng.integers(0, states, size=rows).astype(np.int32)
    ps = params if isinstance(params, list) else [params] * rows
    ps = [dict(p, repetitionWindow=hist_len) for p in ps]
    seeds = [int(rng.integers(1, 2**31)) for _ in range(rows)]
    h = hashlib.sha256()
    for a in (x, hist, hlen) + ((table, mstate) if table is not None else ()):
        h.update(np.ascontiguousarray(a).tobytes())
    return {"name": name, "rows": rows, "vocab": vocab, "softcap": softcap, "params": ps, "seeds": seeds,
            "hist_len": hist_len, "logits": x, "history": hist, "history_len": hlen, "mask_table": table,
            "mask_state": mstate, "sha256": h.hexdigest()}


def case(spec_seed, name, rows, vocab, kind, params, **extra):
    inp = make_inputs(name, spec_seed, rows, vocab, kind, params, **extra)
    x, hist, hlen, table, mstate = inp["logits"], inp["history"], inp["history_len"], inp["mask_table"], inp["mask_state"]
    ps, seeds, softcap, hist_len = inp["params"], inp["seeds"], inp["softcap"], inp["hist_len"]
    rng_state = np.array([seeded_state(s) for s in seeds], dtype=np.float64)
    ids, traces, new_state = O.sample_rows(x, vocab, softcap, hist if hist_len else None, hlen if hist_len else None,
                                           table, mstate, ps, rng_state=rng_state, threads=os.cpu_count() or 1)
    # candidate lists (final, draw order) row by row
    cand_ids, cand_probs, cand_n = [], [], []
    inv = np.float32(1.0 / softcap) if softcap else None
    for r in range(rows):
        row = O.softcap(x[r], softcap) if softcap else x[r].copy()
        if table is not None:
            m = table[mstate[r]]
            bits = (m[np.arange(vocab) >> 5] >> (np.arange(vocab) & 31).astype(np.uint32)) & 1
            row = np.where(bits.astype(bool), row, -np.inf).astype(np.float32)
        res, _ = O.sample_token(row, hist[r, :hist_len] if hist_len else [], ps[r], rng_state=rng_state[r],
                                cand_cap=2048)
        assert res.token == ids[r]
        cand_ids.append(res.candidates)
        cand_probs.append(res.probabilities)
        cand_n.append(res.trace.n_final)  # full count; at most 2048 ids are stored
    cap = max(max(len(c) for c in cand_ids), 1)
    cid = np.full((rows, cap), -1, dtype=np.int32)
    cpr = np.zeros((rows, cap), dtype=np.float64)
    for r in range(rows):
        cid[r, :len(cand_ids[r])] = cand_ids[r]
        cpr[r, :len(cand_probs[r])] = cand_probs[r]
    margins = np.array([[t.margin_top_p, t.margin_draw, t.margin_min_p, t.margin_typical] for t in traces])
    out = {
        f"{name}/rng_state": rng_state, f"{name}/rng_state_after": new_state, f"{name}/ids": ids,
        f"{name}/cand_ids": cid, f"{name}/cand_probs": cpr, f"{name}/cand_count": np.array(cand_n, dtype=np.int32),
        f"{name}/margins": margins,
    }
    meta = {k: inp[k] for k in ("name", "rows", "vocab", "softcap", "params", "seeds", "hist_len", "sha256")}
    meta["mask"] = table is not None
    return out, meta


SPECS = [
    ("c1_small", 8, 8192, "normal", cfg(temperature=0.8, topK=40, topP=0.95), {}),
    ("c2_small", 8, 8192, "zipf", cfg(temperature=1.0, topK=0, topP=0.9, repetitionPenalty=1.1,
                                       presencePenalty=0.5, frequencyPenalty=0.3), {"hist_len": 256}),
    ("c3_small", 16, 8192, "normal", cfg(temperature=0.7, topK=64, topP=0.95, repetitionPenalty=1.1,
                                         presencePenalty=0.5, frequencyPenalty=0.3),
     {"hist_len": 128, "states": 32}),
    ("c4_small", 16, 8192, "normal", cfg(temperature=0.8, topK=50, topP=0.95, repetitionPenalty=1.1,
                                         presencePenalty=0.5, frequencyPenalty=0.3),
     {"hist_len": 64, "states": 32, "density": (0.02, 0.02)}),
    ("c5_small", 8, 8192, "gumbel", cfg(temperature=1.5, topK=1024, topP=0.99), {"ties": 30}),
    ("greedy_penalised", 8, 4096, "normal", cfg(temperature=0, repetitionPenalty=1.3, presencePenalty=0.2,
                                                frequencyPenalty=0.1), {"hist_len": 32}),
    ("min_p", 8, 4096, "normal", cfg(temperature=1.0, topK=200, topP=1, minP=0.05), {}),
    ("typical", 8, 4096, "normal", cfg(temperature=1.0, topK=300, topP=1, typicalP=0.7), {}),
    ("typical_top_p", 8, 4096, "normal", cfg(temperature=0.9, topK=256, topP=0.8, typicalP=0.9,
                                              minP=0.01), {}),
    ("v3", 4, 3, "normal", cfg(temperature=1.0, topK=0, topP=1), {"softcap": 0.0}),
    ("v31_topk_gt_v", 4, 31, "normal", cfg(temperature=0.9, topK=40, topP=0.95), {}),
    ("v1024", 4, 1024, "normal", cfg(temperature=0.8, topK=40, topP=0.95), {}),
    ("v32769", 4, 32769, "normal", cfg(temperature=0.8, topK=100, topP=0.9, repetitionPenalty=1.2),
     {"hist_len": 50}),
    ("flat_ties", 4, 4096, "flat", cfg(temperature=1.0, topK=10, topP=1), {}),
    ("sparse_mask_fill", 8, 4096, "normal", cfg(temperature=1.0, topK=64, topP=1),
     {"states": 8, "density": (0.001, 0.003)}),
    ("neg_inf", 4, 4096, "normal", cfg(temperature=1.0, topK=20, topP=0.9), {"neg_inf": 2000, "softcap": 0.0}),
    ("large_k0_top_p", 4, 16384, "normal", cfg(temperature=1.0, topK=0, topP=0.9), {}),
    ("large_k_big_min_p", 4, 16384, "normal", cfg(temperature=0.6, topK=5000, topP=0.95, minP=0.001), {}),
]


def spec_inputs(index: int):
    """Inputs of SPECS[index] (the seed is 20261201 + index)."""
    name, rows, vocab, kind, params, extra = SPECS[index]
    return make_inputs(name, 20261201 + index, rows, vocab, kind, params, **extra)


def main():
    arrays, metas = {}, []
    for i, (name, rows, vocab, kind, params, extra) in enumerate(SPECS):
        out, meta = case(20261201 + i, name, rows, vocab, kind, params, **extra)
        arrays.update(out)
        metas.append(meta)
        print(name, "ids", out[f"{name}/ids"].tolist())
    arrays["meta_json"] = np.frombuffer(json.dumps(metas).encode(), dtype=np.uint8)
    path = os.path.join(HERE, "config_goldens.npz")
    np.savez_compressed(path, **arrays)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
