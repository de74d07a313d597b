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
    """Batched over leading axes; float32 input is widened to float64."""
    a = np.asarray(logits, dtype=np.float64)
    for _ in range(int(iterations)):
        a = a - _logsumexp(a, -1)
        a = a - _logsumexp(a, -2)
    return np.exp(a)


def _sigmoid(z):
    return 1.0 / (1.0 + np.exp(-z))


def read(x, p, prefix, streams, iterations):
    """Maps and the read value of one block's hyper-connection
    (mhc.py:135-156 compute_mappings, :193-206 read) on streams x [..., S, D]:
    returns (pre [..., S], post [..., S], res [..., S, S]), hidden [..., D]."""
    x = np.asarray(x, dtype=np.float64)
    s, d = streams, x.shape[-1]
    g = lambda n: np.asarray(p[prefix + n], dtype=np.float64)
    flat = x.reshape(*x.shape[:-2], s * d)
    eps = float(np.finfo(np.float32).eps)                 # nn.RMSNorm(eps=None) on fp32
    flat = flat / np.sqrt((flat * flat).mean(-1, keepdims=True) + eps) * g("mapping_norm.weight")
    lg = flat @ g("theta.weight").T
    pre = _sigmoid(g("alpha_pre") * lg[..., :s] + g("pre_bias"))
    post = 2.0 * _sigmoid(g("alpha_post") * lg[..., s:2 * s] + g("post_bias"))
    res = sinkhorn(g("alpha_residual") * lg[..., 2 * s:].reshape(*lg.shape[:-1], s, s)
                   + g("residual_bias"), iterations)
    value = np.einsum("...s,...sd->...d", pre, x)
    mu = value.mean(-1, keepdims=True)
    var = ((value - mu) ** 2).mean(-1, keepdims=True)       # nn.LayerNorm, eps 1e-5
    hidden = (value - mu) / np.sqrt(var + 1e-5) * g("stream_norm.weight") + g("stream_norm.bias")
    return (pre, post, res), hidden


def write(x, update, maps, p, prefix):
    """mhc.py:208-229: x + sigmoid(gating) * scale * (res x + post * update)."""
    x = np.asarray(x, dtype=np.float64)
    _, post, res = maps
    g = lambda n: np.asarray(p[prefix + n], dtype=np.float64)
    mixed = np.einsum("...ij,...jd->...id", res, x) + post[..., None] * np.asarray(update)[..., None, :]
    return x + _sigmoid(g("gating_logit")) * (mixed * g("stream_scale"))
