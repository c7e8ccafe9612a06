"""Constraint bitmask builder (gs_constraint_build_masks) against the oracle on GPU."""
import importlib

import numpy as np
import pytest

import constraint_cases as CC

pytestmark = pytest.mark.gpu

C = importlib.import_module("gemma-webgpu-engine_b200.constraints")


def _gpu(sampler, transitions, finals, tokens, states, term=(), extra=(), mask_words=None):
    dfa = C.Dfa.from_transitions(transitions, finals)
    vb = C.vocab_bytes(tokens)
    g = C.GpuConstraint(sampler, dfa, vb)
    table, dead = g.build_masks(states, termination=term, extra_legal=extra, mask_words=mask_words)
    out = table.cpu().numpy().view(np.uint32), dead.cpu().numpy()
    g.close()
    return out, dfa, vb


@pytest.mark.parametrize("case", CC.kat_cases(), ids=lambda c: c[0])
def test_reference_cases(oracle, sampler, case):
    _, transitions, finals, tokens, checks = case
    states = [s for s, _, _ in checks]
    end = len(tokens) - 1
    (table, dead), dfa, vb = _gpu(sampler, transitions, finals, tokens, states, term=[end])
    node, plen, pb = C.pack_states(states)
    want, wdead = oracle.constraint_masks(dfa.arrays(), vb, node, plen, pb, termination=[end])
    np.testing.assert_array_equal(table, want)
    np.testing.assert_array_equal(dead, wdead)


@pytest.mark.parametrize("seed", range(6))
def test_random_dfas_match_oracle(oracle, sampler, seed):
    transitions, finals, tokens, states, term, extra = CC.random_case(seed)
    W = (len(tokens) + 31) // 32 + 4  # padded rows: the padding words must come back zero
    (table, dead), dfa, vb = _gpu(sampler, transitions, finals, tokens, states, term=term, extra=extra, mask_words=W)
    node, plen, pb = C.pack_states(states)
    want, wdead = oracle.constraint_masks(dfa.arrays(), vb, node, plen, pb, termination=term, extra=extra,
                                          mask_words=W)
    np.testing.assert_array_equal(table, want)
    np.testing.assert_array_equal(dead, wdead)
    assert table.any(), "the case should allow something"


def test_table_feeds_the_sampler(oracle, sampler):
    """Rows built here constrain gs_sample: every sampled id is allowed by its row."""
    import torch
    transitions, finals, tokens, states, term, extra = CC.random_case(11, vocab=4096)
    (table, dead), _, _ = _gpu(sampler, transitions, finals, tokens, states, term=term, extra=extra)
    ok = [i for i in range(len(states)) if not dead[i]]
    rows = len(ok)
    x = torch.randn((rows, len(tokens)), device="cuda") * 3
    p = {"temperature": 1.0, "topK": 40, "topP": 0.95, "minP": 0.0, "typicalP": 1.0, "repetitionPenalty": 1.0,
         "presencePenalty": 0.0, "frequencyPenalty": 0.0, "repetitionWindow": 0}
    t = torch.from_numpy(table.view(np.int32)).cuda()
    res = sampler.sample(x, p, mask_table=t, mask_state=torch.tensor(ok, dtype=torch.int32, device="cuda"),
                         uniforms=torch.rand(rows, dtype=torch.float64, device="cuda"))
    ids = res.ids.cpu().numpy()
    for r, s in enumerate(ok):
        v = int(ids[r])
        assert (int(table[s, v >> 5]) >> (v & 31)) & 1, (s, v)


def test_rejects_bad_inputs(sampler):
    dfa = C.Dfa.from_transitions([[(5, 3, 0)]], [0])  # lo > hi
    with pytest.raises(ValueError, match="lo <= hi"):
        C.GpuConstraint(sampler, dfa, C.vocab_bytes(["a"]))
    g = C.GpuConstraint(sampler, C.Dfa.from_transitions([[(0x61, 0x61, 0)]], [0]), C.vocab_bytes(["a", "b"]))
    with pytest.raises(ValueError, match="node out of range"):
        g.build_masks([3])
    with pytest.raises(ValueError, match="incomplete sequence"):
        g.build_masks([(0, b"\xc3\xa9")])
    g.close()
