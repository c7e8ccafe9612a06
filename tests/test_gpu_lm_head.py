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
