"""Banded (sliding-window) causal attention oracles (numpy).

Two semantics exist in the reference:
  * per-head banded attention with per-head V — fused_banded_local_attention
    (sample_standalone.py:70-85): SDPA with mask j <= t and t - j < window;
  * the CSA local branch (model/layers/csa.py:39-75 prefill, :172-206 decode):
    per-head scores over the causal window, softmax per head, the probabilities
    AVERAGED over heads and applied to one shared d_model-wide value stream.
"""
from __future__ import annotations

import numpy as np


def _fp(x):
    """float32 inputs stay float32 (timed CPU baseline); everything else is float64."""
    x = np.asarray(x)
    return x if x.dtype == np.float32 else x.astype(np.float64)


def _softmax(x, axis=-1):
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=axis, keepdims=True)


def band_mask(t_len: int, window: int) -> np.ndarray:
    i = np.arange(t_len)[:, None]
    j = np.arange(t_len)[None, :]
    return (j <= i) & (i - j < window)


def banded_attention(q, k, v, window: int, scale: float | None = None) -> np.ndarray:
    """q,k [B,T,H,D]; v [B,T,H or 1,Dv] -> [B,T,H,Dv] (sample_standalone.py:70-85)."""
    q, k, v = (_fp(a) for a in (q, k, v))
    b_, t_, h_, d_ = q.shape
    if v.shape[2] == 1 and h_ > 1:
        v = np.broadcast_to(v, (b_, t_, h_, v.shape[-1]))
    scale = 1.0 / np.sqrt(d_) if scale is None else scale
    s = np.einsum("bthd,bshd->bhts", q, k) * scale
    s = np.where(band_mask(t_, window)[None, None], s, -np.inf)
    p = _softmax(s)
    return np.einsum("bhts,bshd->bthd", p, v)


def csa_local(q, k, v_shared, window: int) -> np.ndarray:
    """CSA local branch (csa.py:42-75): q,k [B,T,H,Dh], v_shared [B,T,D] -> [B,T,D].

    window = max(1, min(local_window, T)) as in csa.py:42; probabilities are
    averaged over heads before the shared value product (csa.py:74-75).
    """
    q, k, v = (_fp(a) for a in (q, k, v_shared))
    b_, t_, h_, d_ = q.shape
    w = max(1, min(window, t_))
    s = np.einsum("bthd,bshd->bhts", q, k) / np.sqrt(d_)
    s = np.where(band_mask(t_, w)[None, None], s, -np.inf)
    p = _softmax(s).mean(axis=1)  # [B, T, S]
    return np.einsum("bts,bsd->btd", p, v)


def csa_local_step(q, k_win, v_win, valid=None) -> np.ndarray:
    """CSA decode (csa.py:172-206): q [B,H,Dh]; k_win [B,L,H,Dh]; v_win [B,L,D];
    valid [B,L] bool (history validity).  The caller passes the last
    min(local_window, L) positions, current token last."""
    q, k, v = (_fp(a) for a in (q, k_win, v_win))
    s = np.einsum("bhd,blhd->bhl", q, k) / np.sqrt(q.shape[-1])
    if valid is not None:
        s = np.where(np.asarray(valid)[:, None, :], s, -np.inf)
    p = _softmax(s).mean(axis=1)  # [B, L]
    return np.einsum("bl,bld->bd", p, v)


def csa_layer(hidden, p: dict, n_heads: int, window: int) -> np.ndarray:
    """CompressedSelectiveAttention.forward with the remote branch disabled
    (temporal_compression beyond the sequence): out(local_out(local))."""
    x = _fp(hidden)
    b_, t_, _ = x.shape
    q = (x @ p["query"].T).reshape(b_, t_, n_heads, -1)
    k = (x @ p["key"].T).reshape(b_, t_, n_heads, -1)
    v = x @ p["value"].T
    local = csa_local(q, k, v, window)
    return (local @ p["local_out"].T) @ p["out"].T
