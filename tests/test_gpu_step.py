"""The single-launch decode step (csrc/gs_step.cu) against the oracle.

Batches of at most eight rows whose rows all have topK <= 64 (or temperature 0), with
or without a penalty history (stride <= 512) and a constraint table, run as one kernel: each 2048-id unit keeps
its packs at or above a bound on its k-th best (and its best four), and the last unit of
a row to finish merges the records above a bound on the row's k-th best, then filters
and draws in one warp.  The cases put the row's best values in one unit, across units,
in exact ties and in the partial last unit, and a unit tied throughout (more ties at its
bound than its record holds: its exact best instead); they cover greedy rows, topK
1..64, min-p, typical-p, top-p, the soft cap on and off, -inf logits, bf16,
log-probabilities, calls whose row counts change from call to call (each row's
counter is reset by its last unit), penalty histories, and constrained rows (dense and
sparse masks, fewer allowed ids than topK, a state of -1 and one past the table)."""
from __future__ import annotations

import importlib

import numpy as np
import pytest

import parity_util as PU

pytestmark = pytest.mark.gpu

W = importlib.import_module("gemma-webgpu-engine_b200.workloads")


def _p(**kw):
    p = {"temperature": 0.8, "topK": 40, "topP": 0.95, "minP": 0.0, "typicalP": 1.0, "repetitionPenalty": 1.0,
         "presencePenalty": 0.0, "frequencyPenalty": 0.0, "repetitionWindow": 0}
    p.update(kw)
    return p


def _check(oracle, sampler, x, params, *, softcap=30.0, dtype=None, label="", max_boundary=1, seed=0, cand_cap=64,
           hist=None, hlen=None, table=None, mstate=None):
    rows, V = x.shape
    rng_state = np.array([pkg_seed(seed + r) for r in range(rows)])
    gpu = PU.run_gpu(sampler, x, params, softcap=softcap, rng_state=rng_state, dtype=dtype, cand_cap=cand_cap,
                     history=hist, history_len=hlen, mask_table=table, mask_state=mstate)
    xo = x
    if dtype is not None:
        import torch
        xo = torch.from_numpy(x).to(dtype).float().numpy()
    ids, margins, cands, st = PU.oracle_rows_batched(oracle, xo, V, softcap, params, rng_state=rng_state,
                                                     cand_cap=cand_cap, history=hist, history_len=hlen,
                                                     mask_table=table, mask_state=mstate)
    assert PU.compare(gpu, ids, margins, cands, rng_after=st, label=label) <= max_boundary
    # log-probabilities: tokenLogProbability over the capped logits
    for r in range(rows):
        if gpu.ids[r] >= 0:
            row = oracle.softcap(xo[r], softcap) if softcap else xo[r].astype(np.float32)
            lp = oracle.token_log_probability(row, int(gpu.ids[r]))
            assert abs(gpu.logprob[r] - lp) <= 1e-6 * max(1.0, abs(lp)), (label, r, gpu.logprob[r], lp)
    L = importlib.import_module("gemma-webgpu-engine_b200")._lib
    assert not (gpu.flags & L.FLAG_LARGE_PATH).any(), label
    return gpu


def pkg_seed(s):
    pkg = importlib.import_module("gemma-webgpu-engine_b200")
    return pkg.SeededRandom(s).state


def _rows(rng, rows, V, scale=2.0):
    x = (rng.standard_normal((rows, V)) * scale).astype(np.float32)
    if rows > 1:
        x[1, 1000:1064] = 9.5            # exact ties among the best values, inside one unit
    if rows > 2:
        x[2, ::4099] += 12.0             # the best values spread one per unit
    if rows > 3:
        x[3, -5:] = 11.0                 # the best values in the last unit
    if rows > 4:
        x[4, :] *= 0.01                  # a flat row
    if rows > 5:
        x[5, 2040:2056] = 10.0           # ties across a unit boundary
    if rows > 6:
        x[6, 2048:4096] = 11.0           # a whole unit tied at the top: more ties at the unit's
        #                                  bound than its record holds (the exact-sort fallback)
    return x


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("softcap", [30.0, 0.0], ids=["cap30", "nocap"])
def test_step_rows_and_filters(oracle, sampler, dtype, softcap):
    import torch
    td = torch.bfloat16 if dtype == "bf16" else None
    rng = np.random.default_rng(3 + (dtype == "bf16") + 2 * (softcap == 0))
    V, rows = 262144, 8
    x = _rows(rng, rows, V)
    ps = [_p(temperature=0.0),
          _p(topK=64, topP=1.0),
          _p(topK=1),
          _p(topK=7, minP=0.05),
          _p(topK=40, typicalP=0.8),
          _p(topK=50, topP=0.7, temperature=1.3),
          _p(topK=33, minP=0.01, typicalP=0.9, topP=0.9),
          _p(topK=64, temperature=0.4)]
    _check(oracle, sampler, x, ps, softcap=softcap, dtype=td, label=f"step-{dtype}-{softcap}")


@pytest.mark.parametrize("rows", [1, 2, 3, 5, 8])
def test_step_row_counts_and_counter_reset(oracle, sampler, rows):
    """Calls with changing row counts, back to back: every row's counter must be back at
    zero for the next call (a stale count would merge before the units finish)."""
    rng = np.random.default_rng(100 + rows)
    V = 262144
    for call in range(3):
        x = _rows(rng, rows, V)
        _check(oracle, sampler, x, [_p()], label=f"rows{rows}-call{call}", seed=7 * call)


def test_step_negative_infinity_and_small_vocab(oracle, sampler):
    rng = np.random.default_rng(41)
    V, rows = 262144, 4
    x = (rng.standard_normal((rows, V)) * 2.0).astype(np.float32)
    x[0, rng.choice(V, V // 2, replace=False)] = -np.inf
    x[1, :] = -np.inf
    x[1, 17] = 3.0                       # a single finite id: the rest of the top 40 is -inf
    _check(oracle, sampler, x, [_p(topK=40, topP=1.0)], softcap=0.0, label="neginf")
    for V2 in (2048, 4096, 8192 + 4, 131072):
        x2 = (rng.standard_normal((3, V2)) * 2.0).astype(np.float32)
        _check(oracle, sampler, x2, [_p(topK=min(40, V2), topP=0.9)], label=f"V{V2}", seed=V2)


def test_c1_steps_bit_identical_replay(sampler):
    """The same C1 call twice gives the same bytes (ids, flags, candidates, states)."""
    import torch
    wl = W.make("C1", device="cuda")
    outs = []
    for _ in range(2):
        st = wl.rng_state("cuda")
        r = sampler.sample(wl.logits, wl.params, softcap=wl.softcap, rng_state=st, logprob=True, candidates=40)
        torch.cuda.synchronize()
        outs.append([t.cpu().numpy().tobytes() for t in (r.ids, r.flags, r.logprob, r.cand_ids, r.cand_probs, st)])
    assert outs[0] == outs[1]


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_step_penalty_history(oracle, sampler, dtype):
    """Rows with a penalty history (stride <= 512: the decode default is a 64-id window
    at 1.05): the history ids leave the units' streams and the last CTA scores them
    exactly; histories that are empty, one id, full of repeats, made of the row's best
    ids, and at the stride's limit."""
    import torch
    td = torch.bfloat16 if dtype == "bf16" else None
    rng = np.random.default_rng(57 + (dtype == "bf16"))
    V, rows, H = 262144, 6, 512
    x = _rows(rng, rows, V)
    hist = rng.integers(0, V, (rows, H)).astype(np.int32)
    order = np.argsort(-x, axis=1)
    hist[1, :1] = order[1, :1]                         # the best id only
    hist[2, :64] = order[2, :64]                       # the row's 64 best ids
    hist[3, :200] = np.repeat(order[3, :20], 10)       # twenty ids, ten times each
    hist[4, :] = order[4, :512]                        # the 512 best
    hist[5, ::3] = 7                                   # one id repeated, the rest random
    hlen = np.array([0, 1, 64, 200, 512, 512], dtype=np.int32)
    ps = [_p(temperature=0.0, repetitionPenalty=1.3, repetitionWindow=H),
          _p(topK=40, repetitionPenalty=1.05, repetitionWindow=H),
          _p(topK=64, topP=0.9, repetitionPenalty=1.3, presencePenalty=0.4, frequencyPenalty=0.2, repetitionWindow=H),
          _p(topK=20, minP=0.02, repetitionPenalty=1.2, frequencyPenalty=0.5, repetitionWindow=H),
          _p(topK=50, typicalP=0.9, repetitionPenalty=1.1, presencePenalty=0.5, frequencyPenalty=0.3, repetitionWindow=H),
          _p(temperature=0.0, presencePenalty=2.0, repetitionWindow=H)]
    rng_state = np.array([pkg_seed(900 + r) for r in range(rows)])
    gpu = PU.run_gpu(sampler, x, ps, softcap=30.0, history=hist, history_len=hlen, rng_state=rng_state, dtype=td,
                     cand_cap=64)
    xo = x if td is None else torch.from_numpy(x).to(td).float().numpy()
    ids, margins, cands, st = PU.oracle_rows_batched(oracle, xo, V, 30.0, ps, history=hist, history_len=hlen,
                                                     rng_state=rng_state, cand_cap=64)
    assert PU.compare(gpu, ids, margins, cands, rng_after=st, label=f"step-hist-{dtype}") <= 1
    for r in range(rows):
        lp = oracle.token_log_probability(oracle.softcap(xo[r], 30.0), int(gpu.ids[r]))
        assert abs(gpu.logprob[r] - lp) <= 1e-6 * max(1.0, abs(lp)), (r, gpu.logprob[r], lp)


def test_bound_call_matches_sample(pkg, sampler):
    """GpuSampler.bind (the decode-loop call: structures built once, the logits set per
    call) gives the bytes GpuSampler.sample gives, and refuses logits of another shape."""
    import torch
    lg = torch.stack([W.make("C1", device="cuda", step=s).logits[0] for s in range(6)])
    p = pkg.prepare_params(W.base_params(temperature=0.8, topK=40, topP=0.95, repetitionPenalty=1.05,
                                         repetitionWindow=64))
    hist = torch.randint(0, lg.shape[1], (1, 64), dtype=torch.int32, device="cuda")
    hlen = torch.full((1,), 64, dtype=torch.int32, device="cuda")
    st1 = torch.tensor([pkg.SeededRandom(42).state], dtype=torch.float64, device="cuda")
    st2 = st1.clone()
    step = sampler.bind(lg[0:1], p, softcap=30.0, history=hist, history_len=hlen, rng_state=st1, logprob=True,
                        candidates=40)
    for s in range(6):
        a = step(lg[s:s + 1])
        b = sampler.sample(lg[s:s + 1], p, softcap=30.0, history=hist, history_len=hlen, rng_state=st2,
                           logprob=True, candidates=40)
        torch.cuda.synchronize()
        for x, y in ((a.ids, b.ids), (a.flags, b.flags), (a.logprob, b.logprob), (a.cand_ids, b.cand_ids),
                     (a.cand_probs, b.cand_probs), (a.cand_count, b.cand_count), (st1, st2)):
            assert x.cpu().numpy().tobytes() == y.cpu().numpy().tobytes(), s
    with pytest.raises(ValueError):
        step(lg[0:2])


def _mask(rng, V, dens, extra=()):
    """Allowed-id bitmask rows ([states][V/32] uint32): id 7 always allowed, plus the ids
    in extra[i] for state i."""
    allowed = rng.random((len(dens), V)) < np.array(dens)[:, None]
    allowed[:, 7] = True
    for i, ids in enumerate(extra):
        allowed[i, list(ids)] = True
    bits = allowed.reshape(len(dens), V // 32, 32).astype(np.uint64) << np.arange(32, dtype=np.uint64)
    return bits.sum(axis=-1).astype(np.uint32)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_step_constrained_rows(oracle, sampler, dtype):
    """Rows under a constraint table (the logits of disallowed ids are -inf): a dense mask,
    a sparse one, a row whose state is -1 (no constraint), a state with eleven allowed ids
    for topK 40 and 64 (the rest of the list is the -inf ids in id order: masked ids and
    the row's -inf logits merged), a masked row with a penalty history that names allowed
    and disallowed ids, and greedy rows."""
    import torch
    td = torch.bfloat16 if dtype == "bf16" else None
    rng = np.random.default_rng(71 + (dtype == "bf16"))
    V, rows, H = 262144, 8, 256
    x = _rows(rng, rows, V)
    few = (5000, 70000, 262143, 131072, 2047, 2048, 99, 100, 101, 4095)
    table = _mask(rng, V, [0.3, 0.002, 0.0], extra=((), (), few))
    x[6, 100] = -np.inf                  # an allowed id with a -inf logit, among the masked ones
    mstate = np.array([0, 1, -1, 2, 0, 1, 2, 0], dtype=np.int32)
    hist = np.zeros((rows, H), dtype=np.int32)
    hist[4] = rng.integers(0, V, H)
    hist[4, :32] = np.argsort(-x[4])[:32]  # the row's best ids, allowed or not
    hist[7, :16] = np.array(few + (7, 1, 2, 3, 4, 5))
    hlen = np.array([0, 0, 0, 0, H, 0, 0, 16], dtype=np.int32)
    ps = [_p(topK=40),
          _p(topK=64, topP=0.9),
          _p(topK=40, minP=0.02),
          _p(topK=40, topP=1.0),
          _p(topK=50, repetitionPenalty=1.3, presencePenalty=0.3, frequencyPenalty=0.2, repetitionWindow=H),
          _p(temperature=0.0),
          _p(topK=64, topP=1.0, minP=0.0, typicalP=0.9, temperature=1.2),
          _p(topK=30, repetitionPenalty=1.1, repetitionWindow=H)]
    _check(oracle, sampler, x, ps, dtype=td, hist=hist, hlen=hlen, table=table, mstate=mstate,
           label=f"step-masked-{dtype}", seed=31)
    # every row greedy under the sparse and the eleven-id masks
    g = [_p(temperature=0.0)] * rows
    _check(oracle, sampler, x, g, dtype=td, table=table, mstate=np.array([1, 2, 1, 2, 0, 1, 2, -1], np.int32),
           label=f"step-masked-greedy-{dtype}", seed=5)


def test_step_mask_state_past_table(pkg, sampler):
    """A state at or past the table's rows is an error for that row alone (id -1 and
    GS_FLAG_ERR_INVALID); the host call raises ValueError."""
    import torch
    V = 262144
    x = torch.randn((3, V), device="cuda")
    table = torch.from_numpy(_mask(np.random.default_rng(2), V, [0.5, 0.5]).view(np.int32)).cuda()
    state = torch.tensor([0, 2, 1], dtype=torch.int32, device="cuda")
    u = torch.full((3,), 0.5, dtype=torch.float64, device="cuda")
    r = sampler.sample(x, _p(topK=40), mask_table=table, mask_state=state, uniforms=u)
    flags = r.flags.cpu().numpy().view(np.uint32)
    L = pkg._lib
    assert flags[1] & L.FLAG_ERR_INVALID and int(r.ids[1]) == -1
    for i in (0, 2):
        assert not (flags[i] & L.FLAG_ERRORS)
        assert 0 <= int(r.ids[i]) < V
    with pytest.raises(ValueError, match="mask state"):
        sampler.sample_host(x.cpu().numpy(), _p(topK=40), mask_table=table, mask_state=state.cpu().numpy(),
                            uniforms=np.full(3, 0.5))


def _kernel_names(fn):
    import torch
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]


@pytest.mark.parametrize("case", ["plain", "history", "masked", "masked_history"])
def test_step_is_the_one_launch(sampler, case):
    """Eligible batches (rows <= 8, topK <= 64, history stride <= 512, a constraint table
    or none) run as the one step kernel: no streaming, merge or histogram kernel."""
    import torch
    V, rows = 262144, 4
    x = torch.randn((rows, V), device="cuda")
    kw = {}
    if "history" in case:
        kw["history"] = torch.randint(0, V, (rows, 64), dtype=torch.int32, device="cuda")
        kw["history_len"] = torch.full((rows,), 64, dtype=torch.int32, device="cuda")
    if "masked" in case:
        kw["mask_table"] = torch.from_numpy(_mask(np.random.default_rng(4), V, [0.3]).view(np.int32)).cuda()
        kw["mask_state"] = torch.tensor([0, -1, 0, 0], dtype=torch.int32, device="cuda")
    p = _p(topK=40, repetitionPenalty=1.05, repetitionWindow=64)
    kw["uniforms"] = torch.full((rows,), 0.5, dtype=torch.float64, device="cuda")
    sampler.sample(x, p, **kw)  # warm (plans, attributes)
    names = _kernel_names(lambda: sampler.sample(x, p, **kw))
    ours = [n for n in names if "gs::" in n or "step_kernel" in n or "stream" in n or "finalize" in n]
    if not names:
        pytest.skip("the profiler recorded no CUDA kernels")
    assert any("step_kernel" in n for n in ours), ours
    assert not any(("stream" in n or "finalize" in n or "hist" in n) for n in ours if "step_kernel" not in n), ours
