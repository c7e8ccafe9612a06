"""The constraint-mask restatement against the reference's own legal-set tests
(tests/constraints.spec.ts:27-70), on CPU."""
import importlib

import numpy as np
import pytest

import constraint_cases as CC

C = importlib.import_module("gemma-webgpu-engine_b200.constraints")


def _ids(row, vocab):
    return [v for v in range(vocab) if (int(row[v >> 5]) >> (v & 31)) & 1]


@pytest.mark.parametrize("case", CC.kat_cases(), ids=lambda c: c[0])
def test_reference_legal_sets(oracle, case):
    _, transitions, finals, tokens, checks = case
    dfa = C.Dfa.from_transitions(transitions, finals)
    vb = C.vocab_bytes(tokens)
    node, plen, pb = C.pack_states([s for s, _, _ in checks])
    # termination: a stand-in end token (the last id) shows the accepting rule
    end = len(tokens) - 1
    table, dead = oracle.constraint_masks(dfa.arrays(), vb, node, plen, pb)
    for r, (_, want, _) in enumerate(checks):
        assert _ids(table[r], len(tokens)) == want
        assert dead[r] == (0 if want else 1)
    table, dead = oracle.constraint_masks(dfa.arrays(), vb, node, plen, pb, termination=[end])
    for r, (_, want, accepting) in enumerate(checks):
        expect = sorted(set(want) - {end} | ({end} if accepting else set()))
        assert _ids(table[r], len(tokens)) == expect


def test_extra_ids_join_and_termination_follows_acceptance(oracle):
    _, transitions, finals, tokens, _ = CC.kat_cases()[0]
    dfa = C.Dfa.from_transitions(transitions, finals)
    vb = C.vocab_bytes(tokens)
    node, plen, pb = C.pack_states([0, 2])
    table, dead = oracle.constraint_masks(dfa.arrays(), vb, node, plen, pb, termination=[4], extra=[6, 4])
    assert _ids(table[0], len(tokens)) == [1, 5, 6]  # 4 is a termination id: out unless accepting
    assert _ids(table[1], len(tokens)) == [4, 6]
    assert dead.tolist() == [0, 0]


def test_pack_states_and_vocab_bytes():
    node, plen, pb = C.pack_states([3, (1, b"\xe2\x82")])
    assert node.tolist() == [3, 1] and plen.tolist() == [0, 2]
    assert pb.tolist() == [0, 0, 0, 0xE2, 0x82, 0]
    off, b = C.vocab_bytes([None, "ab", b"\xff", ""])
    assert off.tolist() == [0, 0, 2, 3, 3] and bytes(b) == b"ab\xff"
