"""CUDA path vs the CPU oracle, through the C ABI (libgsampler.so)."""
import json
import math
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import parity_util as PU  # noqa: E402
from golden import make_config_goldens as MG  # noqa: E402

pytestmark = pytest.mark.gpu

SPEC = json.load(open(os.path.join(HERE, "golden", "reference_spec_cases.json")))
GOLD = np.load(os.path.join(HERE, "golden", "config_goldens.npz"))
META = json.loads(bytes(GOLD["meta_json"]).decode())


# ------------------------------------------------------------- reference known answers

@pytest.mark.parametrize("case", SPEC["sample_cases"], ids=[c["name"] for c in SPEC["sample_cases"]])
def test_spec_case_host_buffers(pkg, case):
    """sampleToken known answers through the host-buffer entry point (gs_sample_host)."""
    u = case["uniform"]
    tok = pkg.sample_token(case["logits"], case["history"], case["config"], lambda: u)
    assert tok == case["expect"], case["src"]


@pytest.mark.parametrize("case", SPEC["sample_cases"], ids=[c["name"] for c in SPEC["sample_cases"]])
def test_spec_case_device_buffers(pkg, case):
    import torch
    u = case["uniform"]
    x = torch.tensor(case["logits"], dtype=torch.float32, device="cuda")
    assert pkg.sample_token(x, case["history"], case["config"], lambda: u) == case["expect"], case["src"]


def test_spec_seeded_reproducible(pkg, oracle):
    c = SPEC["reproducible"]
    r1, r2 = pkg.SeededRandom(c["seed"]), pkg.SeededRandom(c["seed"])
    a = [pkg.sample_token(c["logits"], c["history"], c["config"], r1) for _ in range(c["draws"])]
    b = [pkg.sample_token(c["logits"], c["history"], c["config"], r2) for _ in range(c["draws"])]
    assert a == b
    st = oracle.seeded_init(c["seed"])
    ref = []
    for _ in range(c["draws"]):
        res, st = oracle.sample_token(c["logits"], c["history"], c["config"], rng_state=st)
        ref.append(res.token)
    assert a == ref
    assert r1.state == st


def test_spec_log_probability(pkg):
    lp = SPEC["log_probability"]
    for c in lp["cases"]:
        assert abs(pkg.token_log_probability(lp["logits"], c["token"]) - c["expect"]) < 0.005
    with pytest.raises(ValueError, match=lp["error_match"]):
        pkg.token_log_probability(lp["logits"], lp["error_token"])


def test_spec_mask(pkg):
    m = SPEC["mask"]
    out = pkg.mask_constraint_logits(m["logits"], m["legal"], m["termination"]).cpu().numpy()
    assert out.tolist() == [-math.inf if v == "-inf" else v for v in m["expect"]]


def test_build_mask_row(pkg, oracle):
    import torch
    V = 1000
    legal = [1, 3, 31, 32, 999, -5, 1000]
    term = [0, 500]
    row = pkg.build_mask_row(V, legal, term).cpu().numpy().view(np.uint32)
    idx = np.arange(V)
    bits = (row[idx >> 5] >> (idx & 31).astype(np.uint32)) & 1
    ref = oracle.mask_constraint_logits(np.zeros(V, np.float32), legal, term)
    assert (bits == 1).tolist() == (ref == 0).tolist()
    del torch


# ----------------------------------------------------------------- golden configurations

@pytest.mark.parametrize("index", range(len(MG.SPECS)), ids=[s[0] for s in MG.SPECS])
def test_golden_case(sampler, index):
    inp = MG.spec_inputs(index)
    meta = META[index]
    assert inp["sha256"] == meta["sha256"]
    name = inp["name"]
    hl = inp["hist_len"]
    gpu = PU.run_gpu(sampler, inp["logits"], inp["params"], softcap=inp["softcap"],
                     history=inp["history"] if hl else None, history_len=inp["history_len"] if hl else None,
                     mask_table=inp["mask_table"], mask_state=inp["mask_state"],
                     rng_state=GOLD[f"{name}/rng_state"], cand_cap=2048)
    cands = []
    cc = GOLD[f"{name}/cand_count"]
    for r in range(inp["rows"]):
        n = int(cc[r])
        cands.append((GOLD[f"{name}/cand_ids"][r, :n].tolist(), GOLD[f"{name}/cand_probs"][r, :n].tolist(), n))
    margins = GOLD[f"{name}/margins"].min(axis=1)
    diffs = PU.compare(gpu, GOLD[f"{name}/ids"], margins, cands, rng_after=GOLD[f"{name}/rng_state_after"], label=name)
    assert diffs <= max(1, inp["rows"] // 8)


# ------------------------------------------------------------- full-size configurations

def _workload_parity(pkg, oracle, sampler, name, rows, dtype=None, cand=True):
    import torch
    W = pkg.workloads if hasattr(pkg, "workloads") else __import__("importlib").import_module(
        "gemma-webgpu-engine_b200.workloads")
    wl = W.make(name, device="cuda", rows=rows, dtype=dtype)
    x = wl.logits.float().cpu().numpy()
    hist = None if wl.history is None else wl.history.cpu().numpy()
    hlen = None if wl.history_len is None else wl.history_len.cpu().numpy()
    table = None if wl.mask_table is None else wl.mask_table.cpu().numpy().view(np.uint32)
    mstate = None if wl.mask_state is None else wl.mask_state.cpu().numpy()
    rng = wl.rng_state("cpu").numpy()
    gpu = PU.run_gpu(sampler, x, wl.params, softcap=wl.softcap, history=hist, history_len=hlen, mask_table=table,
                     mask_state=mstate, rng_state=rng, cand_cap=2048, dtype=dtype)
    ps = [dict(p, repetitionWindow=(hist.shape[1] if hist is not None else 0)) for p in wl.params]
    ids, margins, cands, st = PU.oracle_rows(oracle, x, wl.vocab, wl.softcap, ps, history=hist, history_len=hlen,
                                             mask_table=table, mask_state=mstate, rng_state=rng, candidates=cand)
    diffs = PU.compare(gpu, ids, margins, cands, rng_after=st, label=name)
    del torch
    return gpu, diffs


def test_c1_full_vocab(pkg, oracle, sampler):
    _workload_parity(pkg, oracle, sampler, "C1", 1)


def test_c1_sequential_steps(pkg, oracle, sampler):
    """C1: 32 sequential steps, fresh logits each step, one SeededRandom stream (seed 42)."""
    import importlib
    import torch
    W = importlib.import_module("gemma-webgpu-engine_b200.workloads")
    st_gpu = torch.tensor([pkg.SeededRandom(42).state], dtype=torch.float64, device="cuda")
    st_ref = oracle.seeded_init(42)
    history = []
    for step in range(32):
        wl = W.make("C1", device="cuda", step=step)
        res = sampler.sample(wl.logits, wl.params, softcap=wl.softcap, rng_state=st_gpu)
        x = wl.logits.cpu().numpy()[0]
        ref, st_ref = oracle.sample_token(oracle.softcap(x, 30.0), history, wl.params[0], rng_state=st_ref)
        assert int(res.ids.item()) == ref.token or (int(res.flags.item()) & 3), f"step {step}"
        history.append(ref.token)
        assert float(st_gpu.item()) == st_ref


def test_c3_constrained(pkg, oracle, sampler):
    _workload_parity(pkg, oracle, sampler, "C3", 24)


def test_c4_full_pipeline_f32(pkg, oracle, sampler):
    _workload_parity(pkg, oracle, sampler, "C4", 24)


def test_c4_full_pipeline_bf16(pkg, oracle, sampler):
    import torch
    _workload_parity(pkg, oracle, sampler, "C4", 16, dtype=torch.bfloat16)


def test_c5_ties_topk1024(pkg, oracle, sampler):
    _workload_parity(pkg, oracle, sampler, "C5", 8)


def test_c2_large_path_top_p_full_vocab(pkg, oracle, sampler):
    _workload_parity(pkg, oracle, sampler, "C2", 8)


# ------------------------------------------------------------------------ properties

@pytest.mark.parametrize("rows", [64, 320], ids=["block-merge", "warp-merge"])
def test_deterministic_replay(pkg, sampler, rows):
    """Two runs on the same inputs give bitwise identical outputs (both merge kernels)."""
    import importlib
    import torch
    W = importlib.import_module("gemma-webgpu-engine_b200.workloads")
    wl = W.make("C4", device="cuda", rows=rows)
    outs = []
    for _ in range(2):
        rng = wl.rng_state("cuda")
        r = sampler.sample(wl.logits, wl.params, softcap=wl.softcap, history=wl.history, history_len=wl.history_len,
                           mask_table=wl.mask_table, mask_state=wl.mask_state, rng_state=rng, logprob=True,
                           candidates=64)
        torch.cuda.synchronize()
        outs.append([t.cpu().numpy().tobytes() for t in (r.ids, r.flags, r.logprob, r.cand_ids, r.cand_probs, rng)])
    assert outs[0] == outs[1]


def test_logprob_matches_oracle(pkg, oracle, sampler):
    import torch
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((4, 50000)) * 3).astype(np.float32)
    gpu = PU.run_gpu(sampler, x, [{"temperature": 0.9, "topK": 20, "topP": 0.9, "minP": 0, "typicalP": 1,
                                  "repetitionPenalty": 1, "presencePenalty": 0, "frequencyPenalty": 0,
                                  "repetitionWindow": 0}], softcap=30.0, uniforms=np.full(4, 0.3), logprob=True)
    for r in range(4):
        ref = oracle.token_log_probability(oracle.softcap(x[r], 30.0), int(gpu.ids[r]))
        assert abs(gpu.logprob[r] - ref) <= 1e-6 * max(1.0, abs(ref))
        t = torch.from_numpy(x[r]).cuda()
        assert abs(pkg.token_log_probability(t, int(gpu.ids[r]), softcap=30.0) - ref) <= 1e-9 * max(1.0, abs(ref))


def test_softcap_matches_oracle_bitwise(pkg, oracle, sampler):
    """The device soft cap equals the host restatement bit for bit over float32 bit
    patterns (all 2^32 of them on hosts with >= 32 cores, else a quarter)."""
    import ctypes
    ncpu = os.cpu_count() or 1
    span = 1 << 28
    starts = range(0, 1 << 32, span) if ncpu >= 32 else range(0, 1 << 32, 4 * span)
    L = pkg._lib.lib()
    for lo in starts:
        d = ctypes.c_uint64(0)
        assert L.gs_softcap_digest(sampler.handle, lo, lo + span, 30.0, ctypes.byref(d)) == 0
        assert d.value == oracle.softcap_digest(lo, lo + span, 30.0), hex(lo)


def test_dead_end_row(pkg, sampler):
    import torch
    V = 4096
    x = torch.randn((2, V), device="cuda")
    table = torch.zeros((2, V // 32), dtype=torch.int32, device="cuda")
    table[1, 0] = 1
    state = torch.tensor([0, 1], dtype=torch.int32, device="cuda")
    p = {"temperature": 1.0, "topK": 10, "topP": 1, "minP": 0, "typicalP": 1, "repetitionPenalty": 1,
         "presencePenalty": 0, "frequencyPenalty": 0, "repetitionWindow": 0}
    r = sampler.sample(x, p, mask_table=table, mask_state=state, uniforms=torch.zeros(2, dtype=torch.float64,
                                                                                     device="cuda"))
    flags = r.flags.cpu().numpy().view(np.uint32)
    assert flags[0] & pkg._lib.FLAG_ERR_DEADEND
    assert int(r.ids[0]) == -1
    assert int(r.ids[1]) == 0 and not (flags[1] & pkg._lib.FLAG_ERRORS)
    with pytest.raises(pkg.SamplerError, match="dead end"):
        sampler.sample_host(x.cpu().numpy(), p, mask_table=table, mask_state=state.cpu().numpy(),
                            uniforms=np.zeros(2))


def test_nonfinite_rejected(pkg, sampler):
    import torch
    x = torch.randn((3, 1000), device="cuda")
    x[0, 17] = float("nan")
    x[1, 900] = float("inf")
    p = {"temperature": 1.0, "topK": 10, "topP": 1, "minP": 0, "typicalP": 1, "repetitionPenalty": 1,
         "presencePenalty": 0, "frequencyPenalty": 0, "repetitionWindow": 0}
    r = sampler.sample(x, p, uniforms=torch.zeros(3, dtype=torch.float64, device="cuda"))
    f = r.flags.cpu().numpy().view(np.uint32)
    assert f[0] & pkg._lib.FLAG_ERR_NONFINITE and f[1] & pkg._lib.FLAG_ERR_NONFINITE
    assert not (f[2] & pkg._lib.FLAG_ERRORS)


def test_empty_logits_and_bad_config(pkg, sampler):
    with pytest.raises(ValueError, match="Cannot sample empty logits"):
        pkg.sample_token([], [], {"temperature": 1.0, "topK": 1, "topP": 1, "minP": 0, "typicalP": 1,
                                  "repetitionPenalty": 1, "presencePenalty": 0, "frequencyPenalty": 0,
                                  "repetitionWindow": 0}, lambda: 0.5)
    with pytest.raises(ValueError, match="topP must be between 0 and 1"):
        pkg.sample_token([1.0, 2.0], [], {"temperature": 1.0, "topK": 1, "topP": 2, "minP": 0, "typicalP": 1,
                                          "repetitionPenalty": 1, "presencePenalty": 0, "frequencyPenalty": 0,
                                          "repetitionWindow": 0}, lambda: 0.5)


def _pack_words(allowed):
    s, v = allowed.shape
    bits = allowed.reshape(s, v // 32, 32).astype(np.uint64) << np.arange(32, dtype=np.uint64)
    return bits.sum(axis=-1).astype(np.uint32)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("k,temp,logprob", [(1, 0.0, False), (1, 0.7, False), (50, 0.8, False), (112, 1.1, False),
                                            (50, 0.8, True)], ids=["greedy", "topk1", "k50", "k112", "k50-logprob"])
def test_stream_tile_modes(pkg, oracle, sampler, dtype, k, temp, logprob):
    """Masks of graded density in one batch (tiles with few allowed ids are gathered
    vector by vector, the others bulk-copied; a requested log-probability reads every
    tile), unmasked rows, a history concentrated in one vocabulary chunk (more penalised
    ids than the per-unit sorted list holds) beside spread-out histories with repeats,
    greedy, topK 1 and the largest topK of the warp-pipelined pass."""
    import torch
    rng = np.random.default_rng(100 + k + (7 if logprob else 0))
    V, rows, H = 65536, 14, 700
    x = (rng.standard_normal((rows, V)) * 2.5).astype(np.float32)
    if dtype == "bf16":
        x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    dens = [0.002, 0.01, 0.03, 0.08, 0.2, 0.5, 1.0]
    allowed = rng.random((len(dens), V)) < np.array(dens)[:, None]
    allowed[:, 7] = True
    table = _pack_words(allowed)
    mstate = np.array([(i % (len(dens) + 1)) - 1 for i in range(rows)], dtype=np.int32)
    hist = np.zeros((rows, H), dtype=np.int32)
    hlen = np.zeros(rows, dtype=np.int32)
    for r in range(rows):
        if r % 3 == 0:
            h = rng.choice(3000, H, replace=False)            # one chunk, > 256 distinct ids
        elif r % 3 == 1:
            h = rng.integers(0, V, H)                           # spread, with repeats
        else:
            h = rng.integers(0, 64, H // 2)                     # few ids, many repeats
        hist[r, :len(h)] = h
        hlen[r] = len(h)
    p = {"temperature": temp, "topK": k, "topP": 0.95, "minP": 0.0, "typicalP": 1.0, "repetitionPenalty": 1.2,
         "presencePenalty": 0.4, "frequencyPenalty": 0.2, "repetitionWindow": H}
    u = rng.random(rows)
    gpu = PU.run_gpu(sampler, x, [p], softcap=30.0, history=hist, history_len=hlen, mask_table=table,
                     mask_state=mstate, uniforms=u, logprob=logprob,
                     dtype=torch.bfloat16 if dtype == "bf16" else None)
    ids, margins, cands, _ = PU.oracle_rows(oracle, x, V, 30.0, [p], history=hist, history_len=hlen,
                                            mask_table=table, mask_state=mstate, uniforms=u)
    diffs = PU.compare(gpu, ids, margins, cands, label=f"tiles-{dtype}-k{k}")
    assert diffs <= 1
    if logprob:
        for r in range(rows):
            ref = oracle.token_log_probability(oracle.softcap(x[r], 30.0), int(gpu.ids[r]))
            assert abs(gpu.logprob[r] - ref) <= 1e-6 * max(1.0, abs(ref)), r


def test_warp_merge_many_rows(pkg, oracle, sampler):
    """Enough rows for the warp-per-row merge (>= 5 per SM on a 148-SM B200), per-row params mixing
    greedy, topK 1..128, min-p, typical-p and top-p, with histories (repeats, masked and
    out-of-range ids) and masks of graded density, including states allowing fewer ids
    than topK (the masked-id filler)."""
    import torch
    rng = np.random.default_rng(77)
    V, rows, H = 32768, 800, 96
    x = (rng.standard_normal((rows, V)) * 2.5).astype(np.float32)
    x[5, 100:140] = 11.0  # exact ties
    dens = [0.0004, 0.003, 0.05, 0.5]
    allowed = rng.random((len(dens), V)) < np.array(dens)[:, None]
    allowed[0] = False
    allowed[0, [3, 77, 4000, 30000]] = True  # 4 allowed ids: fewer than most topK
    table = _pack_words(allowed)
    mstate = np.array([(i % (len(dens) + 2)) - 2 for i in range(rows)], dtype=np.int32)
    hist = rng.integers(-5, V + 5, (rows, H)).astype(np.int32)
    hist[::3, : H // 2] = hist[::3, H // 2:]  # repeats
    hlen = rng.integers(0, H + 1, rows).astype(np.int32)
    ps = []
    for i in range(rows):
        t = [0.0, 0.7, 1.0, 1.3][i % 4]
        ps.append({"temperature": t, "topK": [1, 10, 50, 128][(i // 4) % 4], "topP": [0.9, 1.0, 0.5][i % 3],
                   "minP": [0.0, 0.05][(i // 2) % 2], "typicalP": [1.0, 0.9][(i // 8) % 2],
                   "repetitionPenalty": 1.15, "presencePenalty": 0.3, "frequencyPenalty": 0.1,
                   "repetitionWindow": H})
    u = rng.random(rows)
    gpu = PU.run_gpu(sampler, x, ps, softcap=30.0, history=hist, history_len=hlen, mask_table=table,
                     mask_state=mstate, uniforms=u, cand_cap=128)
    ids, margins, cands, _ = PU.oracle_rows(oracle, x, V, 30.0, ps, history=hist, history_len=hlen,
                                            mask_table=table, mask_state=mstate, uniforms=u, cand_cap=128)
    assert PU.compare(gpu, ids, margins, cands, label="warp-merge") <= 3
    for r in range(rows):
        ref = oracle.token_log_probability(oracle.softcap(x[r], 30.0), int(gpu.ids[r]))
        assert abs(gpu.logprob[r] - ref) <= 1e-6 * max(1.0, abs(ref)), r
    del torch


def test_unaligned_row_stride(pkg, oracle, sampler):
    """Rows whose start is not 16-byte aligned take the scalar path; results unchanged."""
    import torch
    rng = np.random.default_rng(9)
    V = 5001
    x = (rng.standard_normal((4, V)) * 2).astype(np.float32)
    p = {"temperature": 0.8, "topK": 40, "topP": 0.95, "minP": 0, "typicalP": 1, "repetitionPenalty": 1,
         "presencePenalty": 0, "frequencyPenalty": 0, "repetitionWindow": 0}
    u = np.array([0.1, 0.5, 0.7, 0.99])
    gpu = PU.run_gpu(sampler, x, [p], softcap=30.0, uniforms=u)
    ids, margins, cands, _ = PU.oracle_rows(oracle, x, V, 30.0, [p], uniforms=u)
    PU.compare(gpu, ids, margins, cands, label="stride5001")
    del torch
