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


# ------------------------------------------------------------------------
# CSA remote branch (csa.py:77-131 prefill, :208-256 decode step) over the
# causal temporal compressor (compressed_attention.py:85-206), without segment
# ids.  A summary of every complete `ratio`-token block (key = W_k mean, value =
# W_v mean) becomes visible at the block's last position; a query attends to
# its top-k visible summaries per head (softmax over the selected scores,
# renormalised over the visible ones), the heads' results are averaged, and
# remote_out of that is added to the local branch before `out`.
def compress_prefill(hidden, wk, wv, ratio: int):
    """compress(): summaries of the complete blocks and the pending partial
    block.  Returns dict(keys [B,n,W], values [B,n,D], pos [B,n], sum [B,D],
    count [B])."""
    x = _fp(hidden)
    b_, t_, d = x.shape
    n = t_ // ratio
    means = x[:, :n * ratio].reshape(b_, n, ratio, d).mean(2)
    pos = np.broadcast_to((np.arange(n) + 1) * ratio - 1, (b_, n)).copy()
    return dict(keys=means @ _fp(wk).T, values=means @ _fp(wv).T, pos=pos,
                sum=x[:, n * ratio:].sum(1), count=np.full(b_, t_ - n * ratio))


def compress_step(mem, h, wk, wv, ratio: int, position: int):
    """compress_step() + the memory append of forward_step: the token joins the
    pending block; an entry is appended every step, visible (at `position`)
    only when the block completes."""
    h = _fp(h)
    mem["sum"] = mem["sum"] + h
    mem["count"] = mem["count"] + 1
    emitted = mem["count"] >= ratio
    mean = mem["sum"] / np.maximum(mem["count"], 1)[:, None]
    mem["keys"] = np.concatenate([mem["keys"], (mean @ _fp(wk).T)[:, None]], 1)
    mem["values"] = np.concatenate([mem["values"], (mean @ _fp(wv).T)[:, None]], 1)
    mem["pos"] = np.concatenate([mem["pos"], np.where(emitted, position, -1)[:, None]], 1)
    mem["sum"] = np.where(emitted[:, None], 0.0, mem["sum"])
    mem["count"] = np.where(emitted, 0, mem["count"])
    return mem


def remote_attention(q, keys, values, key_pos, query_pos, top_k: int) -> np.ndarray:
    """q [B,T,H,Dh], keys [B,S,H*Dh], values [B,S,D], key_pos [B,S] (-1 =
    not yet visible), query_pos [T]: mean over heads of the top-k visible
    summaries' softmax-weighted values -> [B,T,D]."""
    q = _fp(q)
    b_, t_, h_, dh = q.shape
    out = np.zeros((b_, t_, values.shape[-1]))
    if keys.shape[1] == 0:
        return out
    k = _fp(keys).reshape(b_, -1, h_, dh)
    scores = np.einsum("bthd,bshd->bhts", q, k) / np.sqrt(dh)
    for b in range(b_):
        for t in range(t_):
            vis = np.nonzero((key_pos[b] >= 0) & (key_pos[b] <= query_pos[t]))[0]
            if vis.size == 0:
                continue
            for h in range(h_):
                s = scores[b, h, t, vis]
                order = np.lexsort((vis, -s))[:min(top_k, vis.size)]
                w = _softmax(s[order])
                out[b, t] += w @ _fp(values[b, vis[order]])
    return out / h_


def csa_layer_remote(hidden, p: dict, n_heads: int, window: int, ratio: int, top_k: int):
    """CompressedSelectiveAttention.forward with the remote branch
    (csa.py:39-131): returns (out, compressor memory for decode)."""
    x = _fp(hidden)
    b_, t_, _ = x.shape
    q = (x @ p["query"].T).reshape(b_, t_, n_heads, -1)
    k = (x @ p["key"].T).reshape(b_, t_, n_heads, -1)
    local = csa_local(q, k, x @ p["value"].T, window)
    mem = compress_prefill(x, p["compressor.key"], p["compressor.value"], ratio)
    remote = remote_attention(q, mem["keys"], mem["values"], mem["pos"], np.arange(t_), top_k)
    return (local @ p["local_out"].T + remote @ p["remote_out"].T) @ p["out"].T, mem
