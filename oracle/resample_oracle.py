"""CPU restatement of the device resampler (test infrastructure: only tests import it).

y[c, m] = up * sum_j x[c, j] * h[m * down - j * up + half] over the j where the index lies in
[0, len(h)), inputs outside [0, n) being zero: the zero-phase polyphase FIR that the device kernel
computes (``trc_resample``), written as its defining sum in float64. Pinned against
``scipy.signal.resample_poly`` with the same filter as its ``window`` (a third-party implementation of
the same operation; tests/test_resample.py). The reference itself resamples with soxr, which is not
installed here and whose filter differs: no soxr output is reproduced.
"""

from __future__ import annotations

import numpy as np


def resample(x: np.ndarray, up: int, down: int, h: np.ndarray, n_out: int) -> np.ndarray:
    """x (C, n) -> (C, n_out) float64; h odd-length prototype (without the factor ``up``)."""
    x = np.asarray(x, dtype=np.float64)
    C, n = x.shape
    N = len(h)
    half = (N - 1) // 2
    m = np.arange(n_out, dtype=np.int64)
    t = m * down + half
    j_hi = t // up                       # largest j with t - j * up >= 0
    K = -(-N // up)
    y = np.zeros((C, n_out))
    for k in range(K):                   # j = j_hi - k: filter index t - j * up = (t % up) + k * up
        j = j_hi - k
        idx = (t - j * up)
        ok = (j >= 0) & (j < n) & (idx < N)
        coef = np.where(ok, h[np.minimum(idx, N - 1)], 0.0) * up
        y += coef * x[:, np.clip(j, 0, n - 1)]
    return y


def fold(x: np.ndarray, gains: np.ndarray) -> np.ndarray:
    """(C, n) -> (2, n): the gain matrix applied in float64, channels in order, rounded to float32."""
    x = np.asarray(x, dtype=np.float64)
    y = np.zeros((2, x.shape[1]))
    for k in range(x.shape[0]):
        y += gains[:, k : k + 1] * x[k]
    return y.astype(np.float32)
