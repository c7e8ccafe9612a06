"""The LM-head oracle (oracle_lm_head_shader_f32 / oracle_lm_head_exact) against the
reference's known-answer test for the int2 LM head, and the two evaluations against each
other.

Known answer: tests/qat-linear-gpu.spec.ts:1306-1392 ("projects final activations through
the int2 LM head"): 8 output rows of 96 words, rows filled with 0xaaaaaaaa (codes 2,
weight 0), row 1 0xffffffff (codes 3, weight +1), row 2 0x55555555 (codes 1, weight -1),
row scales [1, 0.5, 0.25, 1, 1, 1, 1, 1], 1536 activations of 1 with sum 1536, output
scale 0 -> logits [0, 768, -384, 0, 0, 0, 0, 0] (toBeCloseTo precision 3 for the
row-major shader).
"""
import numpy as np
import pytest

from oracle import oracle as O

import importlib

LM = importlib.import_module("gemma-webgpu-engine_b200.lm_head")

KAT_EXPECTED = np.array([0, 768, -384, 0, 0, 0, 0, 0], np.float32)


def kat_inputs():
    packed = np.full((8, 96), 0xAAAAAAAA, np.uint32)
    packed[1] = 0xFFFFFFFF
    packed[2] = 0x55555555
    scales = np.array([1, 0.5, 0.25, 1, 1, 1, 1, 1], np.float32)
    return packed, scales, np.ones((1, 1536), np.float32), np.array([1536.0], np.float32)


def test_shader_restatement_matches_known_answer():
    got = O.lm_head(*kat_inputs())[0]
    # toBeCloseTo(expected, 3): |got - expected| < 10^-3 / 2
    assert np.all(np.abs(got - KAT_EXPECTED) < 5e-4)


@pytest.mark.parametrize("in_scale", [0.0, 1.0, 1.0 / 64])
def test_exact_matches_known_answer(in_scale):
    got = O.lm_head(*kat_inputs(), in_scale=in_scale)[0]
    assert np.array_equal(got, KAT_EXPECTED)


def test_code_order():
    # one nonzero code at a time: code j of word w multiplies element 16w + j
    hidden = 256
    packed = np.full((hidden, hidden // 16), 0xAAAAAAAA, np.uint32)
    for e in range(hidden):
        w, j = divmod(e, 16)
        packed[e, w] = (0xAAAAAAAA & ~(3 << (2 * j))) | (3 << (2 * j))  # weight +1 at element e
    act = ((np.arange(hidden) - 128) * 0.5).astype(np.float32)[None, :]  # codes -128..127 at step 0.5
    s = act.sum(dtype=np.float32)
    for in_scale in (None, 0.0, 0.5):
        got = O.lm_head(packed, np.ones(hidden, np.float32), act, [s], in_scale=in_scale)[0]
        assert np.allclose(got, act[0], atol=2e-2), in_scale


@pytest.mark.parametrize("in_scale", [0.02, 0.0])
def test_exact_close_to_shader(in_scale):
    packed, scales, act, act_sum = LM.synthetic(300, 512, rows=3, input_scale=in_scale)
    ref = O.lm_head(packed, scales, act, act_sum)
    ex = O.lm_head(packed, scales, act, act_sum, in_scale=in_scale)
    # both evaluate the same sum; the shader's f32 order errs by at most hidden·eps·Σ|terms|
    codes = ((packed[:, :, None] >> (2 * np.arange(16, dtype=np.uint32))) & 3).reshape(packed.shape[0], -1)
    mag = (codes[None, :, :] * np.abs(act)[:, None, :]).sum(-1) + 2 * np.abs(act_sum)[:, None]
    bound = 512 * np.finfo(np.float32).eps * mag * scales[None, :]
    assert np.all(np.abs(ref - ex) <= bound)


def test_output_srq_grid():
    packed, scales, act, act_sum = LM.synthetic(200, 256, rows=2)
    out = O.lm_head(packed, scales, act, act_sum, out_scale=0.05, in_scale=0.02)
    k = out / np.float32(0.05)
    assert np.all(np.abs(k - np.rint(k)) < 1e-3) and np.all(np.abs(k) <= 128)
