"""maskReasoningLogits restated (src/runtime/gemma-session.ts:1331-1345), on CPU.

The reference has no test of its own for this mask; the cases below state its three
rules: every id whose tokenBytes is null becomes -inf, every other id keeps its raw value,
and with allowEndChannel the end-of-channel id (101) gets its raw value back even when its
bytes are null (a write past a short vocabulary changes nothing)."""
import math

import numpy as np


def test_null_bytes_masked_and_end_channel_restored(oracle):
    V = 128
    x = np.arange(V, dtype=np.float32) * 0.5 - 3.0
    has = np.ones(V, bool)
    has[[0, 1, 2, 100, 101, 127]] = False
    out = oracle.mask_reasoning_logits(x, has, allow_end=False)
    for i in range(V):
        assert (out[i] == x[i]) if has[i] else (out[i] == -math.inf), i
    out = oracle.mask_reasoning_logits(x, has, allow_end=True)
    assert out[101] == x[101]
    assert out[100] == -math.inf and out[0] == -math.inf
    assert np.array_equal(out[102:127], x[102:127])


def test_end_channel_outside_short_vocabulary(oracle):
    x = np.linspace(-1, 1, 50).astype(np.float32)
    has = np.zeros(50, bool)
    has[::3] = True
    a = oracle.mask_reasoning_logits(x, has, allow_end=True)
    b = oracle.mask_reasoning_logits(x, has, allow_end=False)
    assert np.array_equal(a, b)
    assert np.isneginf(a[~has]).all() and np.array_equal(a[has], x[has])


def test_reasoning_state_rule(pkg):
    """Row 1 (end-of-channel allowed) from 16 sampled reasoning tokens on
    (src/runtime/gemma-session.ts:124,676-687)."""
    assert [pkg.reasoning_mask_state(n) for n in (0, 1, 15, 16, 17, 63)] == [0, 0, 0, 1, 1, 1]
