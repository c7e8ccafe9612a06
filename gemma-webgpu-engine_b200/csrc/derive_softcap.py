"""Derivation of the soft-cap polynomial coefficients used by gs_device.cuh and the host
restatement (oracle/oracle.cpp).

  * tanh(a) = a + a^3 * Q(a^2) on [0, 1]: degree-6 Q, fitted for relative error of
    tanh by weighted least squares refined with Lawson reweighting toward minimax.
  * e^r = 1 + r + r^2 * P(r) on [-ln2/2, ln2/2]: degree-4 P, same method (the
    Cody-Waite reduced argument of the |y| >= 1 branch).

Prints the float32 coefficients and the maximum relative error of each fit.  The
committed constants are these values rounded to float32.  The end-to-end error of the
soft cap against c·tanh(x/c) (3.2 ulp, most of it from rounding x·fl(1/c)) and its
monotonicity are checked over every float32 input by the oracle's tests.
"""
import numpy as np


def _lawson(V, r, w, iters):
    W = np.ones(len(r))
    c = None
    for _ in range(iters):
        c, *_ = np.linalg.lstsq(V * (w * np.sqrt(W))[:, None], r * w * np.sqrt(W), rcond=None)
        e = np.abs((V @ c - r) * w)
        W = W * e
        W /= W.sum()
    return c


def fit_tanh(deg=6, n=4000, A=1.0):
    k = np.arange(n)
    x = A * (0.5 - 0.5 * np.cos(np.pi * (k + 0.5) / n))
    x = x[x > 1e-4]
    t = np.tanh(x)
    z = x * x
    r = (t - x) / x ** 3
    w = z / (t / x)
    V = np.vstack([z ** i for i in range(deg + 1)]).T
    c = _lawson(V, r, w, 200)
    return c.astype(np.float32), float(np.max(np.abs((x + x ** 3 * (V @ c)) / t - 1)))


def fit_exp(deg=4, n=4000):
    A = np.log(2) / 2 + 1e-3
    k = np.arange(n)
    x = -A + 2 * A * (0.5 - 0.5 * np.cos(np.pi * (k + 0.5) / n))
    t = np.exp(x)
    r = (t - 1 - x) / x ** 2
    w = x ** 2 / t
    V = np.vstack([x ** i for i in range(deg + 1)]).T
    c = _lawson(V, r, w, 300)
    return c.astype(np.float32), float(np.max(np.abs((1 + x + x ** 2 * (V @ c)) / t - 1)))


if __name__ == "__main__":
    q, eq = fit_tanh()
    p, ep = fit_exp()
    print("tanh Q (z^0..z^6):", q.tolist(), "max rel err", eq)
    print("exp  P (r^0..r^4):", p.tolist(), "max rel err", ep)
