"""The int2 LM head on the GPU (gs_lm_head_logits) against the oracle's exact evaluation,
bit for bit, and against the reference's known-answer test
(tests/qat-linear-gpu.spec.ts:1306-1392, restated in tests/test_oracle_lm_head.py)."""
import importlib

import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
pkg = importlib.import_module("gemma-webgpu-engine_b200")
LM = importlib.import_module("gemma-webgpu-engine_b200.lm_head")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sampler():
    return pkg.GpuSampler(0)


def gpu_logits(sampler, packed, scales, act, act_sum, in_scale, out_scale, pad=0):
    h = LM.GpuLmHead(sampler, packed, scales, in_scale, out_scale)
    try:
        a = torch.from_numpy(np.ascontiguousarray(act)).cuda()
        s = torch.from_numpy(np.ascontiguousarray(act_sum)).cuda()
        V = packed.shape[0]
        buf = torch.full((a.shape[0], V + pad), float("nan"), dtype=torch.float32, device="cuda")
        out = h.logits(a, s, out=buf[:, :V])
        h.check()
        torch.cuda.synchronize()
        if pad:
            assert torch.isnan(buf[:, V:]).all()  # nothing written past the row
        return out.cpu().numpy()
    finally:
        h.close()


@pytest.mark.parametrize("in_scale", [1.0, 1.0 / 64, 0.0])
def test_known_answer(sampler, in_scale):
    packed = np.full((8, 96), 0xAAAAAAAA, np.uint32)
    packed[1] = 0xFFFFFFFF
    packed[2] = 0x55555555
    scales = np.array([1, 0.5, 0.25, 1, 1, 1, 1, 1], np.float32)
    got = gpu_logits(sampler, packed, scales, np.ones((1, 1536), np.float32), np.array([1536.0], np.float32),
                     in_scale, 0.0)
    assert np.array_equal(got[0], np.array([0, 768, -384, 0, 0, 0, 0, 0], np.float32))


CASES = [
    # vocab, hidden, rows, input_scale, output_scale
    (1000, 1536, 1, 0.02, 0.0),
    (4113, 1536, 3, 0.02, 0.05),
    (4096, 256, 64, 0.02, 0.0),
    (2048, 128, 65, 0.015, 0.0),
    (1536, 512, 130, 0.02, 0.1),
    (40000, 1536, 17, 0.02, 0.0),
    (3000, 1536, 300, 0.02, 0.0),
    (777, 1536, 2, 0.0, 0.0),
    (300, 256, 5, 0.0, 0.05),
]


@pytest.mark.parametrize("vocab,hidden,rows,in_scale,out_scale", CASES)
def test_matches_oracle(sampler, vocab, hidden, rows, in_scale, out_scale):
    packed, scales, act, act_sum = LM.synthetic(vocab, hidden, rows, seed=vocab + rows, input_scale=in_scale)
    got = gpu_logits(sampler, packed, scales, act, act_sum, in_scale, out_scale, pad=32)
    want = O.lm_head(packed, scales, act, act_sum, out_scale=out_scale, in_scale=in_scale)
    assert np.array_equal(got, want)


def test_full_vocab(sampler):
    packed, scales, act, act_sum = LM.synthetic(262144, 1536, 2, seed=7)
    got = gpu_logits(sampler, packed, scales, act, act_sum, 0.02, 0.0)
    want = O.lm_head(packed, scales, act, act_sum, in_scale=0.02)
    assert np.array_equal(got, want)


def test_saturated_codes(sampler):
    # activations past the int8 grid clamp to -128 / 127, as srq clamps them
    packed, scales, act, act_sum = LM.synthetic(512, 256, 2, seed=3)
    act = act * 9.0
    got = gpu_logits(sampler, packed, scales, act, act_sum, 0.02, 0.0)
    want = O.lm_head(packed, scales, act, act_sum, in_scale=0.02)
    assert np.array_equal(got, want)


def test_rejects_bad_shapes(sampler):
    packed = np.zeros((64, 10), np.uint32)  # hidden 160: not a multiple of 128
    with pytest.raises(ValueError):
        LM.GpuLmHead(sampler, packed, np.ones(64, np.float32), 0.02)
    packed = np.zeros((64, 112), np.uint32)  # hidden 1792 > 1536
    with pytest.raises(ValueError):
        LM.GpuLmHead(sampler, packed, np.ones(64, np.float32), 0.02)


# ---------------------------------------------------------------- activations -> tokens
from parity_util import compare, oracle_rows  # noqa: E402

C1_PARAMS = dict(temperature=0.8, topK=40, topP=0.95, minP=0.0, typicalP=1.0, repetitionPenalty=1.1,
                 presencePenalty=0.5, frequencyPenalty=0.3)


def _inputs(vocab, rows, seed, in_scale=0.02, hist=16):
    packed, scales, act, act_sum = LM.synthetic(vocab, 1536, rows, seed=seed, input_scale=in_scale)
    g = np.random.default_rng(seed + 1)
    history = g.integers(0, vocab, size=(rows, hist), dtype=np.int64).astype(np.int32)
    history_len = np.full(rows, hist, np.int32)
    rng = np.array([float(1000 + r) for r in range(rows)])
    return packed, scales, act, act_sum, history, history_len, rng


@pytest.mark.parametrize("vocab,rows,topk,masked", [(262144, 1, 40, False), (262144, 3, 40, True), (8192, 20, 50, False),
                                                    (8192, 70, 0, False), (8192, 9, 50, True)])
def test_sample_matches_two_step(sampler, vocab, rows, topk, masked):
    # gs_lm_head_sample == gs_lm_head_logits then gs_sample, bit for bit (with a constraint
    # bitmask of 64 states admitting ~5 % of the ids when `masked`)
    packed, scales, act, act_sum, history, history_len, rng = _inputs(vocab, rows, vocab + rows)
    params = [dict(C1_PARAMS, topK=topk)]
    mk = {}
    if masked:
        g = np.random.default_rng(vocab + 7 * rows)
        allowed = g.random((64, vocab)) < 0.05
        table = np.packbits(allowed, axis=1, bitorder="little").view(np.int32)
        mk = dict(mask_table=torch.from_numpy(np.ascontiguousarray(table)).cuda(),
                  mask_state=torch.from_numpy(g.integers(0, 64, rows).astype(np.int32)).cuda())
    h = LM.GpuLmHead(sampler, packed, scales, 0.02, 0.0)
    try:
        a, s = torch.from_numpy(act).cuda(), torch.from_numpy(act_sum).cuda()
        hi, hl = torch.from_numpy(history).cuda(), torch.from_numpy(history_len).cuda()
        r1 = torch.from_numpy(rng).cuda()
        r2 = r1.clone()
        one = h.sample(a, s, params, softcap=30.0, history=hi, history_len=hl, rng_state=r1, logprob=True,
                       candidates=64, **mk)
        two = sampler.sample(h.logits(a, s), params, softcap=30.0, history=hi, history_len=hl, rng_state=r2,
                             logprob=True, candidates=64, **mk)
        h.check()
        torch.cuda.synchronize()
        exact = ("ids", "flags", "cand_ids", "cand_count")
        if h.fused_calls == 0:  # scratch route: the same kernels on the same logits
            exact += ("logprob", "cand_probs")
        else:  # fused route (one row with a history): normaliser partials summed per block
            np.testing.assert_allclose(one.cand_probs.cpu().numpy(), two.cand_probs.cpu().numpy(), rtol=1e-6, atol=0)
            np.testing.assert_allclose(one.logprob.cpu().numpy(), two.logprob.cpu().numpy(), rtol=1e-9, atol=1e-12)
        for f in exact:
            assert torch.equal(getattr(one, f), getattr(two, f)), f
        assert torch.equal(r1, r2)
    finally:
        h.close()


@pytest.mark.parametrize("rows", [1, 6])
def test_sample_matches_oracle(sampler, rows):
    # the oracle's exact LM head, then the oracle's sampleToken, against one GPU call
    vocab = 262144
    packed, scales, act, act_sum, history, history_len, rng = _inputs(vocab, rows, 77 + rows)
    params = [C1_PARAMS]
    logits = O.lm_head(packed, scales, act, act_sum, in_scale=0.02)
    ids, margins, cands, st = oracle_rows(O, logits, vocab, 30.0, [dict(C1_PARAMS, repetitionWindow=history.shape[1])],
                                          history=history, history_len=history_len, rng_state=rng)
    h = LM.GpuLmHead(sampler, packed, scales, 0.02, 0.0)
    try:
        r = torch.from_numpy(rng).cuda()
        res = h.sample(torch.from_numpy(act).cuda(), torch.from_numpy(act_sum).cuda(), params, softcap=30.0,
                       history=torch.from_numpy(history).cuda(), history_len=torch.from_numpy(history_len).cuda(),
                       rng_state=r, logprob=True, candidates=2048)
        torch.cuda.synchronize()
    finally:
        h.close()
    from parity_util import GpuOut
    gpu = GpuOut(ids=res.ids.cpu().numpy(), flags=res.flags.cpu().numpy().view(np.uint32), rng_after=r.cpu().numpy(),
                 cand_ids=res.cand_ids.cpu().numpy(), cand_probs=res.cand_probs.cpu().numpy(),
                 cand_count=res.cand_count.cpu().numpy(), logprob=res.logprob.cpu().numpy())
    compare(gpu, ids, margins, cands, rng_after=st, label="lm_head_sample")


# ---------------------------------------------------------------- fused route (no history)
NOHIST = dict(C1_PARAMS, repetitionPenalty=1.0, presencePenalty=0.0, frequencyPenalty=0.0)


def _mask(vocab, rows, seed, density=0.05, states=64):
    g = np.random.default_rng(seed)
    allowed = g.random((states, vocab)) < density
    allowed = np.pad(allowed, ((0, 0), (0, -vocab % 128)))  # whole 16-byte groups of words
    table = np.packbits(allowed, axis=1, bitorder="little").view(np.uint32)
    return np.ascontiguousarray(table), g.integers(0, states, rows).astype(np.int32)


def _gpu_out(res, r):
    from parity_util import GpuOut
    return GpuOut(ids=res.ids.cpu().numpy(), flags=res.flags.cpu().numpy().view(np.uint32), rng_after=r.cpu().numpy(),
                  cand_ids=res.cand_ids.cpu().numpy(), cand_probs=res.cand_probs.cpu().numpy(),
                  cand_count=res.cand_count.cpu().numpy(), logprob=res.logprob.cpu().numpy())


@pytest.mark.parametrize("vocab,rows,topk,masked,hidden,out_scale", [
    (262144, 1, 40, False, 1536, 0.0), (262144, 2, 64, True, 1536, 0.0), (262144, 2, 1, False, 1536, 0.0),
    (5000, 2, 40, False, 1536, 0.0), (8192, 2, 20, True, 1536, 0.0), (40000, 2, 40, False, 256, 0.0),
    (100000, 2, 30, False, 640, 0.05), (262144, 1, 40, False, 1536, 0.05), (5000, 1, 40, True, 1536, 0.0),
    (3000, 1, 64, False, 1536, 0.0)])
def test_fused_matches_oracle(sampler, vocab, rows, topk, masked, hidden, out_scale):
    # activations -> tokens through the fused route (the logits never stored) against the
    # oracle's exact LM head and sampleToken on the same inputs (hidden 256 and 640: other
    # chunk splits of the dot products; output srq on; one row: the shards' records
    # combined in the kernel, by the bound or, with fewer shards than topK, the radix select)
    packed, scales, act, act_sum = LM.synthetic(vocab, hidden, rows, seed=vocab + 3 * rows + topk, input_scale=0.02)
    rng = np.array([float(5000 + r) for r in range(rows)])
    params = [dict(NOHIST, topK=topk)]
    table, state = _mask(vocab, rows, vocab + rows) if masked else (None, None)
    logits = O.lm_head(packed, scales, act, act_sum, out_scale=out_scale, in_scale=0.02)
    ids, margins, cands, st = oracle_rows(O, logits, vocab, 30.0, [dict(params[0], repetitionWindow=0)],
                                          mask_table=table, mask_state=state, rng_state=rng)
    h = LM.GpuLmHead(sampler, packed, scales, 0.02, out_scale, route="fused")
    try:
        r = torch.from_numpy(rng).cuda()
        mk = {} if table is None else dict(mask_table=torch.from_numpy(table.view(np.int32)).cuda(),
                                           mask_state=torch.from_numpy(state).cuda())
        res = h.sample(torch.from_numpy(act).cuda(), torch.from_numpy(act_sum).cuda(), params, softcap=30.0,
                       rng_state=r, logprob=True, candidates=2048, **mk)
        h.check()
        torch.cuda.synchronize()
        assert h.fused_calls == 1
    finally:
        h.close()
    compare(_gpu_out(res, r), ids, margins, cands, rng_after=st, label="lm_head_fused")


@pytest.mark.parametrize("rows,temperature,topk,masked", [(1, 0.8, 40, False), (2, 0.8, 64, True), (1, 0.0, 40, False),
                                                          (2, 0.0, 10, True), (1, 1.3, 5, True)])
def test_fused_matches_two_step(sampler, rows, temperature, topk, masked):
    # fused route == gs_lm_head_logits + gs_sample: ids, candidate ids and counts and flags
    # exactly; probabilities and log-probabilities to float64 summation order
    vocab = 262144
    packed, scales, act, act_sum = LM.synthetic(vocab, 1536, rows, seed=91 + rows, input_scale=0.02)
    params = [dict(NOHIST, temperature=temperature, topK=topk)]
    mk = {}
    if masked:
        table, state = _mask(vocab, rows, 17 + rows, density=0.3)
        mk = dict(mask_table=torch.from_numpy(table.view(np.int32)).cuda(), mask_state=torch.from_numpy(state).cuda())
    h = LM.GpuLmHead(sampler, packed, scales, 0.02, 0.0, route="fused")
    try:
        a, s = torch.from_numpy(act).cuda(), torch.from_numpy(act_sum).cuda()
        r1 = torch.tensor([float(70 + i) for i in range(rows)], dtype=torch.float64, device="cuda")
        r2 = r1.clone()
        one = h.sample(a, s, params, softcap=30.0, rng_state=r1, logprob=True, candidates=64, **mk)
        two = sampler.sample(h.logits(a, s), params, softcap=30.0, rng_state=r2, logprob=True, candidates=64, **mk)
        h.check()
        torch.cuda.synchronize()
        assert h.fused_calls == 1
        for f in ("ids", "flags", "cand_ids", "cand_count"):
            assert torch.equal(getattr(one, f), getattr(two, f)), f
        assert torch.equal(r1, r2)
        np.testing.assert_allclose(one.cand_probs.cpu().numpy(), two.cand_probs.cpu().numpy(), rtol=1e-6, atol=0)
        np.testing.assert_allclose(one.logprob.cpu().numpy(), two.logprob.cpu().numpy(), rtol=1e-9, atol=1e-12)
    finally:
        h.close()


def test_fused_error_rows_and_routes(sampler):
    # rows the fused route cannot sample flag as the two-step route flags them (a mask
    # state past the table, every logit NaN); batches outside its scope take the scratch route
    vocab = 8192
    packed, scales, act, act_sum = LM.synthetic(vocab, 1536, 2, seed=5, input_scale=0.02)
    table, state = _mask(vocab, 2, 9, states=8)
    L = pkg._lib
    h = LM.GpuLmHead(sampler, packed, scales, 0.02, 0.0, route="fused")
    try:
        a = torch.from_numpy(act).cuda()
        for case in ("state", "nan"):
            sums, st = act_sum.copy(), state.copy()
            if case == "state":
                st[1] = 8  # past the table
            else:
                sums[1] = np.nan
            s = torch.from_numpy(sums).cuda()
            mk = dict(mask_table=torch.from_numpy(table.view(np.int32)).cuda(), mask_state=torch.from_numpy(st).cuda())
            params = [dict(NOHIST, topK=40)]
            r1 = torch.arange(2, dtype=torch.float64, device="cuda")
            r2 = r1.clone()
            one = h.sample(a, s, params, softcap=30.0, rng_state=r1, logprob=True, candidates=64, **mk)
            two = sampler.sample(h.logits(a, s), params, softcap=30.0, rng_state=r2, logprob=True, candidates=64, **mk)
            torch.cuda.synchronize()
            for f in ("ids", "flags", "cand_count"):
                assert torch.equal(getattr(one, f), getattr(two, f)), (case, f)
            fl = one.flags.cpu().numpy().view(np.uint32)
            assert fl[1] & L.FLAG_ERRORS and not (fl[0] & L.FLAG_ERRORS), case
        assert h.fused_calls == 2
        # three rows, a penalty history, topK past 64: the scratch route
        s = torch.from_numpy(act_sum).cuda()
        packed3, scales3, act3, sum3 = LM.synthetic(vocab, 1536, 3, seed=6, input_scale=0.02)
        h.sample(torch.from_numpy(act3).cuda(), torch.from_numpy(sum3).cuda(), [dict(NOHIST, topK=40)], softcap=30.0,
                 rng_state=torch.zeros(3, dtype=torch.float64, device="cuda"))
        hist = torch.zeros((2, 4), dtype=torch.int32, device="cuda")
        h.sample(a, s, [C1_PARAMS], softcap=30.0, history=hist,
                 history_len=torch.full((2,), 4, dtype=torch.int32, device="cuda"),
                 rng_state=torch.zeros(2, dtype=torch.float64, device="cuda"))
        h.sample(a, s, [dict(NOHIST, topK=100)], softcap=30.0, rng_state=torch.zeros(2, dtype=torch.float64, device="cuda"))
        torch.cuda.synchronize()
        assert h.fused_calls == 2
    finally:
        h.close()


def test_route_choice(sampler):
    # auto: the two-step route where gs_sample takes the single-launch decode step (no
    # history, or one of at most 512 ids), the fused route for one row with a longer
    # history; "two-step" never fuses; both routes give the same ids
    vocab = 262144
    packed, scales, act, act_sum = LM.synthetic(vocab, 1536, 1, seed=12, input_scale=0.02)
    a, s = torch.from_numpy(act).cuda(), torch.from_numpy(act_sum).cuda()
    g = np.random.default_rng(3)
    long_hist = torch.from_numpy(g.integers(0, vocab, (1, 1024)).astype(np.int32)).cuda()
    short_hist = long_hist[:, :256].contiguous()
    h = LM.GpuLmHead(sampler, packed, scales, 0.02, 0.0)
    try:
        assert h.route == "auto"
        ids = {}
        for route, hist, fused in (("auto", None, 0), ("auto", short_hist, 0), ("auto", long_hist, 1),
                                   ("two-step", long_hist, 0), ("fused", None, 1)):
            h.set_route(route)
            before = h.fused_calls
            kw = {} if hist is None else dict(history=hist, history_len=torch.tensor([hist.shape[1]], dtype=torch.int32,
                                                                                       device="cuda"))
            res = h.sample(a, s, [C1_PARAMS], softcap=30.0, rng_state=torch.tensor([9.0], dtype=torch.float64,
                                                                                   device="cuda"), **kw)
            torch.cuda.synchronize()
            assert h.fused_calls - before == fused, (route, None if hist is None else hist.shape[1])
            ids.setdefault(None if hist is None else hist.shape[1], set()).add(int(res.ids[0]))
        assert all(len(v) == 1 for v in ids.values()), ids
        with pytest.raises(ValueError):
            h.set_route("fastest")
    finally:
        h.close()


@pytest.mark.parametrize("topk,masked,temperature", [(40, False, 0.8), (64, True, 0.8), (40, False, 0.0), (5, True, 1.2)])
def test_fused_history_matches_oracle(sampler, topk, masked, temperature):
    # one row with a penalty history (repeated ids, the row's best ids, a negative id, ids
    # masked out) through the fused route against the oracle
    vocab = 262144
    packed, scales, act, act_sum = LM.synthetic(vocab, 1536, 1, seed=400 + topk, input_scale=0.02)
    logits = O.lm_head(packed, scales, act, act_sum, in_scale=0.02)
    order = np.argsort(-logits[0], kind="stable")
    g = np.random.default_rng(topk)
    hist = np.concatenate([order[:3], order[:1], order[5:8], [-5], g.integers(0, vocab, 20)]).astype(np.int32)
    history, history_len = hist[None, :].copy(), np.array([len(hist)], np.int32)
    params = [dict(C1_PARAMS, temperature=temperature, topK=topk)]
    table, state = _mask(vocab, 1, 77, density=0.5) if masked else (None, None)
    rng = np.array([123.0])
    ids, margins, cands, st = oracle_rows(O, logits, vocab, 30.0, [dict(params[0], repetitionWindow=len(hist))],
                                          history=history, history_len=history_len, mask_table=table,
                                          mask_state=state, rng_state=rng)
    h = LM.GpuLmHead(sampler, packed, scales, 0.02, 0.0, route="fused")
    try:
        r = torch.from_numpy(rng).cuda()
        mk = {} if table is None else dict(mask_table=torch.from_numpy(table.view(np.int32)).cuda(),
                                           mask_state=torch.from_numpy(state).cuda())
        res = h.sample(torch.from_numpy(act).cuda(), torch.from_numpy(act_sum).cuda(), params, softcap=30.0,
                       history=torch.from_numpy(history).cuda(), history_len=torch.from_numpy(history_len).cuda(),
                       rng_state=r, logprob=True, candidates=2048, **mk)
        h.check()
        torch.cuda.synchronize()
        assert h.fused_calls == 1
    finally:
        h.close()
    compare(_gpu_out(res, r), ids, margins, cands, rng_after=st, label="lm_head_fused_history")
