"""Constraint bitmask tables built on the GPU from a compiled DFA.

The reference compiles a generation constraint (regex / JSON / JSON Schema) into a DFA
over Unicode code points (src/runtime/constraints.ts:175-220, with refa) and, at every
decode step, walks the vocabulary's token-byte trie from the current constraint state to
list the legal token ids (legalTokenIds, :56-92).  The sampler here consumes a bitmask
table [states, V/32] and a per-row state index instead; this module builds the table's
rows for any set of constraint states at once (gs_constraint_build_masks): the DFA and
the token bytes are uploaded once, and each state's row is the legal set of
selectConstrainedToken (src/runtime/gemma-session.ts:1315-1326).

The DFA is given in the form of a refa DFA node's transition map: per node, sorted
disjoint code-point ranges (lo, hi inclusive) with their target nodes, and the accepting
nodes.  Compiling regexes or schemas to that form stays with the host (out of scope).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Iterable, Sequence

import numpy as np

from . import _lib
from .sampling import SamplerError


@dataclass
class Dfa:
    """Per-node code-point ranges: node n's transitions are rows
    range_offsets[n]:range_offsets[n+1] of (range_lo, range_hi, range_target)."""
    range_offsets: np.ndarray
    range_lo: np.ndarray
    range_hi: np.ndarray
    range_target: np.ndarray
    final: np.ndarray

    @property
    def nodes(self) -> int:
        return len(self.final)

    @classmethod
    def from_transitions(cls, transitions: Sequence[Iterable[tuple[int, int, int]]], finals: Iterable[int]) -> "Dfa":
        """`transitions[n]` lists (lo, hi, target) for node n (code points, hi inclusive);
        the ranges are sorted here and must not overlap."""
        off, lo, hi, tgt = [0], [], [], []
        for ranges in transitions:
            for a, b, t in sorted(ranges):
                lo.append(a)
                hi.append(b)
                tgt.append(t)
            off.append(len(lo))
        fin = np.zeros(len(transitions), np.uint8)
        for n in finals:
            fin[n] = 1
        return cls(np.array(off, np.int32), np.array(lo, np.uint32), np.array(hi, np.uint32),
                   np.array(tgt, np.int32), fin)

    def arrays(self):
        return (self.range_offsets, self.range_lo, self.range_hi, self.range_target, self.final)


def vocab_bytes(tokens: Sequence[bytes | str | None]) -> tuple[np.ndarray, np.ndarray]:
    """(offsets [V+1] int64, bytes uint8) of a vocabulary given as its tokens' bytes (str is
    UTF-8 encoded; None or b"" is a token without bytes, never legal)."""
    parts = [b"" if t is None else (t.encode("utf-8") if isinstance(t, str) else bytes(t)) for t in tokens]
    off = np.zeros(len(parts) + 1, np.int64)
    off[1:] = np.cumsum([len(p) for p in parts])
    return off, np.frombuffer(b"".join(parts), np.uint8).copy()


def pack_states(states: Sequence[tuple[int, bytes]] | Sequence[int]):
    """(node, pending_len, pending_bytes[3·S]) of constraint states given as node ids or
    (node, pending UTF-8 bytes) pairs."""
    nodes, plen, pb = [], [], []
    for s in states:
        n, pend = (s, b"") if isinstance(s, (int, np.integer)) else (s[0], bytes(s[1]))
        if len(pend) > 3:
            raise ValueError("at most 3 pending UTF-8 bytes")
        nodes.append(int(n))
        plen.append(len(pend))
        pb.extend(list(pend) + [0] * (3 - len(pend)))
    return np.array(nodes, np.int32), np.array(plen, np.uint8), np.array(pb, np.uint8)


class GpuConstraint:
    """A DFA and a vocabulary resident on the sampler's device (gs_constraint_create)."""

    def __init__(self, sampler, dfa: Dfa, vocab: tuple[np.ndarray, np.ndarray]):
        self._L = _lib.lib()
        self._keep = [np.ascontiguousarray(a) for a in dfa.arrays()]
        off, lo, hi, tgt, fin = self._keep
        d = _lib.GsDfaDesc(dfa.nodes, off.ctypes.data, lo.ctypes.data, hi.ctypes.data, tgt.ctypes.data,
                           fin.ctypes.data)
        voff = np.ascontiguousarray(vocab[0], np.int64)
        vb = np.ascontiguousarray(vocab[1], np.uint8)
        if vb.size == 0:
            vb = np.zeros(1, np.uint8)
        v = _lib.GsVocabBytesDesc(len(voff) - 1, voff.ctypes.data, vb.ctypes.data)
        self.vocab = len(voff) - 1
        self.device = sampler.device
        self._h = ctypes.c_void_p()
        st = self._L.gs_constraint_create(sampler.handle, ctypes.byref(d), ctypes.byref(v), ctypes.byref(self._h))
        if st != _lib.GS_OK:
            msg = self._L.gs_last_error(sampler.handle)
            raise (ValueError if st == _lib.GS_EINVAL else SamplerError)(
                *(((msg or b"").decode(),) if st == _lib.GS_EINVAL else (st, (msg or b"").decode())))

    def close(self):
        if self._h:
            self._L.gs_constraint_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def build_masks(self, states, termination: Sequence[int] = (), extra_legal: Sequence[int] = (),
                    mask_words: int | None = None, table=None, stream=None):
        """Rows of the bitmask table (an int32 device tensor [S, mask_words], bit v of a
        row: token v allowed) and the per-state dead-end flags (int32 device tensor) for
        `states` (node ids, or (node, pending UTF-8 bytes) pairs)."""
        import torch
        node, plen, pb = pack_states(states)
        S = len(node)
        W = mask_words or (self.vocab + 31) // 32
        dev = torch.device("cuda", self.device)
        if table is None:
            table = torch.empty((S, W), dtype=torch.int32, device=dev)
        dead = torch.empty(S, dtype=torch.int32, device=dev)
        term = np.ascontiguousarray(termination, np.int32)
        extra = np.ascontiguousarray(extra_legal, np.int32)
        if stream is None:
            stream = torch.cuda.current_stream(dev).cuda_stream
        st = self._L.gs_constraint_build_masks(
            self._h, S, node.ctypes.data, plen.ctypes.data, pb.ctypes.data, term.ctypes.data if term.size else None,
            term.size, extra.ctypes.data if extra.size else None, extra.size, ctypes.c_void_p(table.data_ptr()), W,
            ctypes.c_void_p(dead.data_ptr()), ctypes.c_void_p(stream))
        if st != _lib.GS_OK:
            msg = (self._L.gs_constraint_last_error(self._h) or b"").decode()
            raise (ValueError(msg) if st == _lib.GS_EINVAL else SamplerError(st, msg))
        return table, dead
