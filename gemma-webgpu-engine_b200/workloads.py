"""Seeded synthetic inputs for the five benchmark configurations (V = 262144).

No public dataset is involved: the configurations are defined by their distributions.
All tensors are generated with torch's counter-based (Philox) generator on the target
device from fixed seeds, so a workload is reproducible on one software stack; parity
tests copy the same bytes to the host for the CPU oracle instead of regenerating them.

  C1  B=1, N(0,4), soft cap 30, T=0.8, topK 40, topP 0.95, seed 42, 256 sequential steps
  C2  B=64, N(0,4) + Zipf(s=1.1) bias bias[perm[r]] = -1.1·ln(r+1), soft cap 30,
      1024 uniform history ids (window 1024), penalties 1.1/0.5/0.3, T=1, topK 0, topP 0.9,
      seeds 1000+row
  C3  B=256, N(0,4), soft cap 30, 4096 DFA states each admitting a seeded 1-5% of ids
      (at least one), uniform state per row, 512 uniform history ids (window 512,
      penalties 1.1/0.5/0.3), T=0.7, topK 64, topP 0.95, seeds 2000+row
  C4  B=4096, N(0,4), soft cap 30, 256 history ids at 1.1/0.5/0.3, 4096 states at 2%,
      T=0.8, topK 50, topP 0.95, seeds 3000+row; float32 and bfloat16 logits
  C5  B=8, Gumbel(0, beta=2) + 30 planted exact ties per row (set to the row maximum),
      T=1.5, topK 1024, topP 0.99, seeds 4000+row; vocabulary split in 8 shards
"""
from __future__ import annotations

from dataclasses import dataclass, field

VOCAB = 262144
SOFTCAP = 30.0


def base_params(**kw) -> dict:
    from .decoding import DEFAULT_DECODING_CONFIG
    p = dict(DEFAULT_DECODING_CONFIG)
    p.update(kw)
    return p


@dataclass
class Workload:
    name: str
    logits: object                  # [rows, vocab] device tensor (raw, before the soft cap)
    params: list                    # DecodingConfig dicts (one, or one per row)
    softcap: float = SOFTCAP
    history: object = None          # [rows, H] int32 (already windowed)
    history_len: object = None      # [rows] int32
    mask_table: object = None       # [states, vocab/32] int32
    mask_state: object = None       # [rows] int32
    seeds: list = field(default_factory=list)
    vocab: int = VOCAB

    @property
    def rows(self) -> int:
        return self.logits.shape[0]

    def rng_state(self, device):
        import torch
        from .sampling import SeededRandom
        return torch.tensor([SeededRandom(s).state for s in self.seeds], dtype=torch.float64, device=device)

    def algorithmic_bytes_per_row(self) -> int:
        """Bytes a row must move at least: logits + constraint bitmask row + history ids."""
        b = self.vocab * self.logits.element_size()
        if self.mask_table is not None:
            b += self.vocab // 8
        if self.history is not None:
            b += 4 * self.history.shape[1]
        return b


def _gen(device, seed):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def normal_logits(rows, vocab, device, seed, std=2.0):
    import torch
    return torch.randn((rows, vocab), generator=_gen(device, seed), device=device, dtype=torch.float32) * std


def uniform_history(rows, length, vocab, device, seed):
    import torch
    h = torch.randint(0, vocab, (rows, length), generator=_gen(device, seed), device=device, dtype=torch.int64)
    return h.to(torch.int32), torch.full((rows,), length, dtype=torch.int32, device=device)


def pack_bits(allowed):
    """bool [S, V] -> int32 [S, V/32] little-endian bit words."""
    import torch
    S, V = allowed.shape
    w = allowed.view(S, V // 32, 32).to(torch.int64)
    shifts = torch.arange(32, device=allowed.device, dtype=torch.int64)
    words = (w << shifts).sum(dim=-1)
    words = torch.where(words >= 2**31, words - 2**32, words)
    return words.to(torch.int32)


def dfa_mask_table(states, vocab, device, seed, lo=0.01, hi=0.05, chunk=256):
    """States x vocab allowed-token bitmask: state s admits a seeded fraction in [lo, hi]
    of ids (density drawn per state), and at least one id."""
    import torch
    g = _gen(device, seed)
    density = lo + (hi - lo) * torch.rand(states, generator=g, device=device)
    forced = torch.randint(0, vocab, (states,), generator=g, device=device)
    out = torch.empty((states, vocab // 32), dtype=torch.int32, device=device)
    for s0 in range(0, states, chunk):
        s1 = min(states, s0 + chunk)
        allowed = torch.rand((s1 - s0, vocab), generator=g, device=device) < density[s0:s1, None]
        allowed[torch.arange(s1 - s0, device=device), forced[s0:s1]] = True
        out[s0:s1] = pack_bits(allowed)
    return out


def make(name: str, device="cuda", rows: int | None = None, vocab: int = VOCAB, step: int = 0,
         dtype=None, shard: int = 0) -> Workload:
    """Builds configuration `name` (C1..C5).  `rows` overrides the batch (tests use fewer
    rows of the same distribution); `step` selects the fresh logits of a C1 step; `shard`
    (C4) gives another GPU's batch of the same distribution: its own logits, histories,
    states and row seeds, the constraint table shared (shard 0 is the batch itself)."""
    import torch
    if name == "C1":
        r = rows or 1
        logits = normal_logits(r, vocab, device, seed=step)
        p = base_params(temperature=0.8, topK=40, topP=0.95, seed=42, repetitionWindow=0)
        wl = Workload("C1", logits, [p], seeds=[42] * r, vocab=vocab)
    elif name == "C2":
        r = rows or 64
        g = _gen(device, 11)
        perm = torch.randperm(vocab, generator=g, device=device)
        bias = torch.empty(vocab, device=device, dtype=torch.float32)
        bias[perm] = -1.1 * torch.log(torch.arange(1, vocab + 1, device=device, dtype=torch.float64)).to(torch.float32)
        logits = normal_logits(r, vocab, device, seed=12) + bias[None, :]
        hist, hlen = uniform_history(r, 1024, vocab, device, seed=13)
        ps = [base_params(temperature=1.0, topK=0, topP=0.9, repetitionPenalty=1.1, presencePenalty=0.5,
                          frequencyPenalty=0.3, repetitionWindow=1024, seed=1000 + i) for i in range(r)]
        wl = Workload("C2", logits, ps, history=hist, history_len=hlen, seeds=[1000 + i for i in range(r)],
                      vocab=vocab)
    elif name == "C3":
        r = rows or 256
        logits = normal_logits(r, vocab, device, seed=21)
        table = dfa_mask_table(4096, vocab, device, seed=22)
        state = torch.randint(0, 4096, (r,), generator=_gen(device, 23), device=device, dtype=torch.int64).to(torch.int32)
        hist, hlen = uniform_history(r, 512, vocab, device, seed=24)
        ps = [base_params(temperature=0.7, topK=64, topP=0.95, repetitionPenalty=1.1, presencePenalty=0.5,
                          frequencyPenalty=0.3, repetitionWindow=512, seed=2000 + i) for i in range(r)]
        wl = Workload("C3", logits, ps, history=hist, history_len=hlen, mask_table=table, mask_state=state,
                      seeds=[2000 + i for i in range(r)], vocab=vocab)
    elif name == "C4":
        r = rows or 4096
        o = 1000 * shard
        logits = normal_logits(r, vocab, device, seed=31 + o)
        table = dfa_mask_table(4096, vocab, device, seed=32, lo=0.02, hi=0.02)
        state = torch.randint(0, 4096, (r,), generator=_gen(device, 33 + o), device=device,
                              dtype=torch.int64).to(torch.int32)
        hist, hlen = uniform_history(r, 256, vocab, device, seed=34 + o)
        p = base_params(temperature=0.8, topK=50, topP=0.95, repetitionPenalty=1.1, presencePenalty=0.5,
                        frequencyPenalty=0.3, repetitionWindow=256)
        wl = Workload("C4", logits, [p], history=hist, history_len=hlen, mask_table=table, mask_state=state,
                      seeds=[3000 + shard * r + i for i in range(r)], vocab=vocab)
    elif name == "C5":
        r = rows or 8
        g = _gen(device, 41)
        u = torch.rand((r, vocab), generator=g, device=device, dtype=torch.float64).clamp_(1e-300, 1 - 1e-16)
        logits = (-2.0 * torch.log(-torch.log(u))).to(torch.float32)
        ties = torch.stack([torch.randperm(vocab, generator=g, device=device)[:30] for _ in range(r)])
        rowmax = logits.max(dim=1, keepdim=True).values
        logits.scatter_(1, ties, rowmax.expand(r, 30))
        p = base_params(temperature=1.5, topK=1024, topP=0.99, repetitionWindow=0)
        wl = Workload("C5", logits, [p], seeds=[4000 + i for i in range(r)], vocab=vocab)
    else:
        raise ValueError(f"unknown workload {name}")
    if dtype is not None:
        wl.logits = wl.logits.to(dtype)
    return wl


def synthetic_token_bytes(vocab: int = VOCAB, seed: int = 51):
    """(offsets, bytes) of a seeded stand-in for a SentencePiece vocabulary's token bytes
    (the Gemma tokenizer's bytes are not available here): lengths 1-16 bytes (mean about
    6), mostly ASCII letters, digits, punctuation and a leading space, about 15 % of the
    tokens with 2-4-byte UTF-8 characters, and 256 single raw-byte tokens at the front."""
    import numpy as np
    rng = np.random.default_rng(seed)
    ascii_pool = np.frombuffer(b" abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789.,:;\"'{}[]()-_",
                               dtype=np.uint8)
    parts = [bytes([b]) for b in range(256)]
    lens = np.clip(rng.geometric(0.18, vocab - 256), 1, 16)
    for n in lens.tolist():
        if rng.random() < 0.15:
            s = ""
            while len(s.encode("utf-8")) < n:
                r = rng.random()
                cp = int(rng.integers(0x80, 0x800)) if r < 0.5 else int(rng.integers(0x800, 0xD800)) if r < 0.9 \
                    else int(rng.integers(0x10000, 0x20000))
                s += chr(cp)
            parts.append(s.encode("utf-8"))
        else:
            parts.append(ascii_pool[rng.integers(0, len(ascii_pool), n)].tobytes())
    off = np.zeros(vocab + 1, np.int64)
    off[1:] = np.cumsum([len(x) for x in parts])
    return off, np.frombuffer(b"".join(parts), np.uint8).copy()


def synthetic_dfa(nodes: int = 4096, seed: int = 52):
    """A seeded code-point DFA standing in for a compiled grammar: a third of the nodes
    are string interiors (every character except '"' and '\\' loops back; '"' leaves),
    the rest have 1-8 ranges of ASCII or other Unicode characters to random nodes; a fifth
    of the nodes accept.  Returns the transitions and the accepting nodes, the input of
    constraints.Dfa.from_transitions."""
    import numpy as np
    rng = np.random.default_rng(seed)
    transitions = []
    for n in range(nodes):
        if n % 3 == 0:
            out = int(rng.integers(0, nodes))
            transitions.append([(0x20, 0x21, n), (0x22, 0x22, out), (0x23, 0x5B, n), (0x5D, 0x10FFFF, n)])
            continue
        cuts, ranges, last = set(), [], -1
        for _ in range(int(rng.integers(1, 9))):
            if rng.random() < 0.8:
                lo = int(rng.integers(0x20, 0x7F))
                hi = min(0x7E, lo + int(rng.integers(0, 12)))
            else:
                lo = int(rng.integers(0x80, 0x30000))
                hi = lo + int(rng.integers(0, 5000))
            cuts.add((lo, hi))
        for lo, hi in sorted(cuts):
            if lo <= last:
                continue
            ranges.append((lo, hi, int(rng.integers(0, nodes))))
            last = hi
        transitions.append(ranges)
    finals = [n for n in range(nodes) if rng.random() < 0.2]
    return transitions, finals
