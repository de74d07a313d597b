"""Gated DeltaNet recurrence, chunked form and layer (numpy oracle).

Reference: model/layers/gated_deltanet.py
  * step (:140-149): carry <- 0 where reset; pred = k^T S; delta = v - pred;
    S <- decay * S + beta * k delta^T; out = (q^T S) * gate (S is the UPDATED state)
  * projections and gates (:125-132): q,k L2-normalised per head with
    rsqrt(max(sum x^2, 1e-12)); beta = sigmoid(beta_proj(x)) (with bias);
    gate = sigmoid(gate_proj(x)); decay = sigmoid(decay_logit[h]) per head
  * causal depthwise conv gate on the block input (:56-78, :254-276), then
    out = out_proj(o) * sigmoid(conv).
"""
from __future__ import annotations

import numpy as np


def _fp(x):
    """float32 inputs stay float32 (timed CPU baseline); everything else is float64."""
    x = np.asarray(x)
    return x if x.dtype == np.float32 else x.astype(np.float64)


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-_fp(x)))


def l2norm_heads(x: np.ndarray) -> np.ndarray:
    """x * rsqrt(max(sum(x^2), 1e-12)) over the last dim (gated_deltanet.py:128-129)."""
    x = _fp(x)
    return x / np.sqrt(np.maximum((x * x).sum(-1, keepdims=True), 1e-12))


def gdn_recurrent(q, k, v, beta, gate, reset, alpha, state):
    """Sequential scan of gated_deltanet.py:140-149.

    q,k [B,T,H,K]; v,gate [B,T,H,V]; beta [B,T,H] (already sigmoided);
    reset [B,T] bool or None; alpha: decay per head [H] (the reference's
    sigmoid(decay_logit)) or per token [B,T,H]; state [B,H,K,V].
    Returns out [B,T,H,V] (= (q^T S_t) * gate_t) and the final state, float64.
    """
    q, k, v, gate = (_fp(a) for a in (q, k, v, gate))
    beta = _fp(beta)
    if beta.ndim == 4:
        beta = beta[..., 0]
    b_, t_, h_, _ = q.shape
    alpha = _fp(alpha)
    alpha = np.broadcast_to(alpha if alpha.ndim == 3 else alpha[None, None, :], (b_, t_, h_))
    s = np.array(_fp(state), copy=True)
    out = np.empty(v.shape, dtype=v.dtype)
    for t in range(t_):
        if reset is not None:
            s[np.asarray(reset)[:, t]] = 0.0
        kt, vt = k[:, t], v[:, t]
        pred = np.einsum("bhk,bhkv->bhv", kt, s)
        delta = vt - pred
        s = alpha[:, t, :, None, None] * s + beta[:, t, :, None, None] * np.einsum("bhk,bhv->bhkv", kt, delta)
        out[:, t] = np.einsum("bhk,bhkv->bhv", q[:, t], s) * gate[:, t]
    return out, s


def gdn_chunked(q, k, v, beta, gate, reset, log_alpha, state, chunk: int = 64):
    """Chunk-parallel form of the same recurrence (used to check the kernel's algebra).

    With w_t = beta_t (v_t - S_{t-1}^T k_t) the recurrence is
    S_t = alpha_t S_{t-1} + k_t w_t^T, hence inside a chunk with cumulative
    decay Gamma_t = prod_{j<=t} alpha_j:
        S_t = Gamma_t S_0 + sum_{i<=t} (Gamma_t/Gamma_i) k_i w_i^T
        (I + A) W = diag(beta) V - diag(beta Gamma_{t-1}) K S_0,
        A[t,i] = beta_t (Gamma_{t-1}/Gamma_i) k_t.k_i  (i < t)
        O = diag(Gamma) Q S_0 + (M o Q K^T) W,  M[t,i] = Gamma_t/Gamma_i (i <= t)
        S_C = Gamma_C S_0 + (diag(Gamma_C/Gamma_i) K)^T W.
    A reset at token r drops S_0 and every earlier token for t >= r (segment
    masks).  log_alpha is [H] or [B,T,H]; everything in float64.
    """
    q, k, v, gate = (_fp(a) for a in (q, k, v, gate))
    beta = _fp(beta)
    if beta.ndim == 4:
        beta = beta[..., 0]
    b_, t_, h_, kd = q.shape
    la = _fp(log_alpha)
    la = np.broadcast_to(la if la.ndim == 3 else la[None, None, :], (b_, t_, h_))
    rs = np.zeros((b_, t_), dtype=bool) if reset is None else np.asarray(reset, dtype=bool)
    s = np.array(_fp(state), copy=True)
    out = np.empty(v.shape, dtype=v.dtype)
    for c0 in range(0, t_, chunk):
        c1 = min(t_, c0 + chunk)
        n = c1 - c0
        for b in range(b_):
            seg = np.cumsum(rs[b, c0:c1])
            same = seg[:, None] == seg[None, :]
            first = seg == 0
            for h in range(h_):
                kc, qc, vc, bc = k[b, c0:c1, h], q[b, c0:c1, h], v[b, c0:c1, h], beta[b, c0:c1, h]
                g = np.cumsum(la[b, c0:c1, h])
                gprev = g - la[b, c0:c1, h]
                tri = np.tril(np.ones((n, n), dtype=bool), -1)
                a = bc[:, None] * np.exp(gprev[:, None] - g[None, :]) * (kc @ kc.T)
                a = np.where(tri & same, a, 0.0)
                tinv = np.linalg.inv(np.eye(n) + a)
                s0 = s[b, h]
                rhs = bc[:, None] * vc - (bc * np.exp(gprev) * first)[:, None] * (kc @ s0)
                w = tinv @ rhs
                m = np.where(np.tril(np.ones((n, n), dtype=bool)) & same,
                             np.exp(g[:, None] - g[None, :]), 0.0)
                o = (np.exp(g) * first)[:, None] * (qc @ s0) + (m * (qc @ kc.T)) @ w
                out[b, c0:c1, h] = o * gate[b, c0:c1, h]
                last = seg == seg[-1]
                kt = kc * (np.exp(g[-1] - g) * last)[:, None]
                s[b, h] = (np.exp(g[-1]) if seg[-1] == 0 else 0.0) * s0 + kt.T @ w
    return out, s


def causal_conv(hidden, weight, reset=None, history=None):
    """Depthwise causal conv (kernel K, no bias) over [B,T,D] (gated_deltanet.py:56-78).

    weight [D,1,K] or [D,K].  Without history the sequence is left-padded with
    zeros; a reset at t masks taps that reach before t (same segment only).
    With history [B,K-1,D] (decode, :257-268) the taps read the history
    (zeroed for rows whose reset flag is set).
    """
    x = _fp(hidden)
    w = _fp(weight).reshape(x.shape[-1], -1)
    kk = w.shape[1]
    b_, t_, d_ = x.shape
    if history is not None:
        hist = _fp(history)
        if reset is not None:
            hist = np.where(np.asarray(reset)[:, 0][:, None, None], 0.0, hist)
        full = np.concatenate([hist[:, -(kk - 1):], x], axis=1)
        out = np.zeros_like(x)
        for j in range(kk):
            out += full[:, j:j + t_] * w[None, None, :, j]
        return out
    pad = np.concatenate([np.zeros((b_, kk - 1, d_)), x], axis=1)
    seg = np.zeros((b_, t_), dtype=np.int64) if reset is None else np.cumsum(np.asarray(reset), axis=1)
    seg_pad = np.concatenate([np.full((b_, kk - 1), -1), seg], axis=1)
    out = np.zeros_like(x)
    masked = reset is not None and bool(np.asarray(reset)[:, 1:].any())
    for j in range(kk):
        tap = pad[:, j:j + t_]
        if masked:
            tap = tap * (seg_pad[:, j:j + t_] == seg)[..., None]
        out += tap * w[None, None, :, j]
    return out


def gdn_layer(hidden, p: dict, state, reset=None, conv_history=None):
    """GatedDeltaNet.forward (gated_deltanet.py:119-276) with weights in dict p.

    p keys: q_proj, k_proj, v_proj, beta_proj, beta_bias, gate_proj, out_proj,
    conv [D,1,4], decay_logit [H]; heads/key_dim/value_dim from shapes.
    Returns (out [B,T,D], final state [B,H,K,V]).
    """
    x = _fp(hidden)
    b_, t_, _ = x.shape
    h_ = p["decay_logit"].shape[0]
    q = (x @ p["q_proj"].T).reshape(b_, t_, h_, -1)
    k = (x @ p["k_proj"].T).reshape(b_, t_, h_, -1)
    v = (x @ p["v_proj"].T).reshape(b_, t_, h_, -1)
    q, k = l2norm_heads(q), l2norm_heads(k)
    beta = sigmoid(x @ p["beta_proj"].T + p["beta_bias"])
    gate = sigmoid(x @ p["gate_proj"].T).reshape(b_, t_, h_, -1)
    decay = sigmoid(p["decay_logit"])
    o, s = gdn_recurrent(q, k, v, beta, gate, reset, decay, state)
    conv = causal_conv(x, p["conv"], reset, conv_history)
    out = (o.reshape(b_, t_, -1) @ p["out_proj"].T) * sigmoid(conv)
    return out, s
