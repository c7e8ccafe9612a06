"""The reasoning-channel mask (maskReasoningLogits, src/runtime/gemma-session.ts:1331-1345)
as a two-row bitmask table on GPU, against the oracle's restatement."""
import numpy as np
import pytest

import parity_util as PU

pytestmark = pytest.mark.gpu

V = 262144


def _has_bytes(seed):
    """A vocabulary where the special ids (0-2, 100-105, a scattered 1 %) have null bytes."""
    rng = np.random.default_rng(seed)
    has = rng.random(V) > 0.01
    has[[0, 1, 2, 100, 101, 102, 103, 104, 105]] = False
    return has


def test_rows_match_oracle_masks(pkg, oracle, sampler):
    has = _has_bytes(1)
    rows = pkg.reasoning_mask_rows(has, sampler=sampler).cpu().numpy().view(np.uint32)
    idx = np.arange(V)
    x = np.zeros(V, np.float32)
    for r, allow in ((0, False), (1, True)):
        bits = ((rows[r][idx >> 5] >> (idx & 31).astype(np.uint32)) & 1).astype(bool)
        ref = np.isfinite(oracle.mask_reasoning_logits(x, has, allow_end=allow))
        assert np.array_equal(bits, ref), r


def test_required_reasoning_steps_match_oracle(pkg, oracle, sampler):
    """24 steps of a required-reasoning channel (C1's filters, penalties on over the
    history, fresh logits each step, one seeded stream): before 16 reasoning tokens the
    end-of-channel id stays masked, from then on it is allowed; GPU ids, candidates and
    PRNG states follow the oracle sampling the masked copy of the logits."""
    import torch
    has = _has_bytes(2)
    table = pkg.reasoning_mask_rows(has, sampler=sampler)
    rng = np.random.default_rng(3)
    cfg = {"temperature": 0.8, "topK": 40, "topP": 0.95, "minP": 0.0, "typicalP": 1.0, "repetitionPenalty": 1.1,
           "presencePenalty": 0.5, "frequencyPenalty": 0.3, "repetitionWindow": 64}
    st_gpu = torch.tensor([pkg.SeededRandom(7).state], dtype=torch.float64, device="cuda")
    st_ref = oracle.seeded_init(7)
    history = list(rng.integers(0, V, 20))
    for step in range(24):
        x = (rng.standard_normal(V) * 2.0).astype(np.float32)
        x[101] = 12.0  # the end-of-channel id would win whenever it is allowed
        state = pkg.reasoning_mask_state(step)
        h = pkg.windowed_history(history, cfg["repetitionWindow"])
        ht = torch.tensor([h], dtype=torch.int32, device="cuda")
        res = sampler.sample(torch.from_numpy(x[None]).cuda(), cfg, history=ht,
                             history_len=torch.tensor([len(h)], dtype=torch.int32, device="cuda"),
                             mask_table=table, mask_state=torch.tensor([state], dtype=torch.int32, device="cuda"),
                             rng_state=st_gpu, candidates=40)
        masked = oracle.mask_reasoning_logits(x, has, allow_end=bool(state))
        ref, st_ref = oracle.sample_token(masked, h, cfg, rng_state=st_ref, cand_cap=40)
        tok = int(res.ids.item())
        flagged = bool(int(res.flags.item()) & pkg._lib.FLAG_BOUNDARY) or \
            min(ref.trace.margin_top_p, ref.trace.margin_draw) < PU.BOUNDARY
        assert tok == ref.token or flagged, f"step {step}"
        if not flagged:
            n = int(res.cand_count.item())
            assert res.cand_ids[0, :n].cpu().tolist() == ref.candidates, step
        assert (101 in ref.candidates) == (state == 1), step
        assert float(st_gpu.item()) == st_ref
        history.append(ref.token)
