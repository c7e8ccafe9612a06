"""The soft cap's stated properties, over every positive float32 input (the routine is
odd, so this covers all of them): monotone, and within 3.2 ulp of c·tanh(x/c).  The CUDA
routine is compared with this one bit for bit by the GPU tests (a digest over all 2^32
bit patterns)."""
import numpy as np


def test_softcap_monotone_and_accurate_everywhere(oracle):
    max_ulp, decreases = oracle.softcap_check(30.0)
    assert decreases == 0
    assert max_ulp <= 3.25, max_ulp


def test_softcap_is_odd_and_saturates(oracle):
    x = np.array([0.0, 1e-20, 3.0, 29.999998, 30.0, 45.0, 269.9, 270.0, 1e30, np.inf], dtype=np.float32)
    y = oracle.softcap(x, 30.0)
    assert np.array_equal(oracle.softcap(-x, 30.0), -y)
    assert y[-1] == 30.0 and y[-2] == 30.0
    assert np.all(np.diff(y) >= 0)
