"""Test infrastructure: numpy restatement of the mHC mapping normaliser.

Reference: model/layers/mhc.py:12-17 (_sinkhorn_impl): starting from the
logits (fp32), `iterations` rounds of subtracting the log-sum-exp over the last
axis (rows), then over the second-to-last axis (columns); the result is exp of
that.  Computed here in float64.  Pinned to outputs of the reference function
itself (tests/golden/make_engine_ops.py).
"""
from __future__ import annotations

import numpy as np


def _logsumexp(a: np.ndarray, axis: int) -> np.ndarray:
    m = np.max(a, axis=axis, keepdims=True)
    return m + np.log(np.sum(np.exp(a - m), axis=axis, keepdims=True))


def sinkhorn(logits: np.ndarray, iterations: int = 20) -> np.ndarray:
    a = np.asarray(logits, dtype=np.float32).astype(np.float64)
    for _ in range(int(iterations)):
        a = a - _logsumexp(a, -1)
        a = a - _logsumexp(a, -2)
    return np.exp(a)
