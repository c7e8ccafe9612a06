"""DFA / vocabulary cases shared by the constraint-mask tests.

The known-answer cases restate the three legal-set tests of the reference
(tests/constraints.spec.ts:27-70) with their DFAs written out by hand: the minimal DFA of
each regex over code points (the form refa produces; refa itself is JavaScript and does
not run here).  The random cases cover split and invalid UTF-8, pending states, and
extra / termination ids.
"""
from __future__ import annotations

import numpy as np


def kat_cases():
    """[(name, transitions, finals, tokens, [(state, expected legal ids, accepting)])]"""
    a_bc = ("a(?:b|c)", [[(0x61, 0x61, 1)], [(0x62, 0x63, 2)], []], [2],
            [None, "a", "b", "c", "ab", "ac", "x"],
            [(0, [1, 4, 5], False), (1, [2, 3], False), (2, [], True)])
    arabic = "أ".encode("utf-8")  # D8 A3
    alif = ("أ", [[(0x623, 0x623, 1)], []], [1],
            [None, arabic[:1], arabic[1:], arabic, b"\xff"],
            [(0, [1, 3], False), ((0, arabic[:1]), [2], False), (1, [], True)])
    brace = ("\\{", [[(0x7B, 0x7B, 1)], []], [1],
             [None, b"\xef", b"\xbf", b"\xbd", "{"],
             [(0, [4], False)])
    return [a_bc, alif, brace]


def _encode(cp: int) -> bytes:
    return chr(cp).encode("utf-8", "surrogatepass")


def random_case(seed: int, nodes: int = 40, vocab: int = 3000):
    rng = np.random.default_rng(seed)
    spans = [(0x20, 0x7E), (0x80, 0x7FF), (0x800, 0xFFFF), (0x10000, 0x10FFFF)]
    transitions = []
    for _ in range(nodes):
        cuts = set()
        k = int(rng.integers(0, 7))
        for _ in range(k):
            a, b = spans[int(rng.choice(4, p=[0.55, 0.2, 0.15, 0.1]))]
            lo = int(rng.integers(a, b + 1))
            hi = min(b, lo + int(rng.integers(0, 40 if a < 0x80 else 4000)))
            cuts.add((lo, hi))
        ranges, last = [], -1
        for lo, hi in sorted(cuts):
            if lo <= last:
                continue
            ranges.append((lo, hi, int(rng.integers(0, nodes))))
            last = hi
        transitions.append(ranges)
    finals = [n for n in range(nodes) if rng.random() < 0.2] or [0]
    tokens = []
    for _ in range(vocab):
        kind = rng.random()
        if kind < 0.03:
            tokens.append(None)
            continue
        parts = b""
        for _ in range(int(rng.integers(1, 5))):
            r = rng.random()
            if r < 0.6:
                parts += bytes([int(rng.integers(0x20, 0x7F))])
            elif r < 0.92:
                a, b = spans[int(rng.integers(1, 4))]
                cp = int(rng.integers(a, b + 1))
                if 0xD800 <= cp <= 0xDFFF:
                    cp = 0x41
                parts += _encode(cp)
            else:
                parts += bytes([int(rng.integers(0x80, 0x100))])
        cut = rng.random()
        if cut < 0.15 and len(parts) > 1:  # a token that splits a UTF-8 sequence
            i = int(rng.integers(1, len(parts)))
            parts = parts[:i] if rng.random() < 0.5 else parts[i:]
        tokens.append(parts)
    states = []
    for _ in range(24):
        n = int(rng.integers(0, nodes))
        r = rng.random()
        if r < 0.6:
            states.append(n)
        else:
            lead = int(rng.choice([0xC3, 0xD8, 0xE0, 0xE2, 0xED, 0xF0, 0xF4]))
            pend = bytes([lead])
            need = 2 if lead <= 0xDF else 3 if lead <= 0xEF else 4
            while len(pend) < need - 1 and rng.random() < 0.7:
                pend += bytes([int(rng.integers(0x80, 0xC0))])
            states.append((n, pend))
    term = [int(x) for x in rng.choice(vocab, 3, replace=False)]
    extra = [int(x) for x in rng.choice(vocab, 4, replace=False)]
    return transitions, finals, tokens, states, term, extra
