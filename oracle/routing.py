"""Router top-k, dispatch plan and routed SwiGLU experts (numpy oracle).

Reference: model/layers/context_router.py:72-74 (top-k over fp32 logits,
softmax of the selected values) and model/layers/moe.py:29-82
(_moe_dispatch_fused: sort routes by expert, bincount, offsets, SwiGLU experts,
probability-weighted index_add).
"""
from __future__ import annotations

import numpy as np


def router_topk(logits: np.ndarray, k: int, bias: np.ndarray | None = None):
    """Top-k ordered by (value desc, index asc) and softmax of the k values.

    context_router.py:73-74.  torch.topk leaves tie order unspecified; this
    oracle (and the kernel) break ties by the lower expert index.
    Returns (idx int64 [N,k], prob float64 [N,k]).
    """
    x = np.asarray(logits, dtype=np.float32)
    if bias is not None:
        x = (x + np.asarray(bias, dtype=np.float32)[None, :]).astype(np.float32)
    n, e = x.shape
    cols = np.broadcast_to(np.arange(e), (n, e))
    order = np.lexsort((cols, -x), axis=-1)  # primary: value desc, secondary: index asc
    idx = order[:, :k].astype(np.int64)
    vals = np.take_along_axis(x, idx, axis=-1).astype(np.float64)
    vals = vals - vals[:, :1]
    ex = np.exp(vals)
    prob = ex / ex.sum(axis=-1, keepdims=True)
    return idx, prob


def dispatch_plan(idx: np.ndarray, n_experts: int, tile_m: int = 128) -> dict[str, np.ndarray]:
    """Stable expert-grouped order of the flat routes r = t*k + s (moe.py:42-60).

    moe.py sorts with torch.sort (unstable); the stable order is the one the
    kernel reproduces bit-exactly.
    """
    idx = np.asarray(idx, dtype=np.int64)
    n, k = idx.shape
    flat = idx.reshape(-1)
    order = np.argsort(flat, kind="stable").astype(np.int64)
    counts = np.bincount(flat, minlength=n_experts).astype(np.int64)
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    tiles = (counts + tile_m - 1) // tile_m
    tile_offsets = np.concatenate([[0], np.cumsum(tiles)]).astype(np.int64)
    route_pos = np.empty(n * k, dtype=np.int64)
    route_pos[order] = np.arange(n * k)
    return dict(counts=counts, offsets=offsets, tile_offsets=tile_offsets, sort_order=order,
                perm_token=order // k, route_pos=route_pos)


def append_shared(plan: dict, idx: np.ndarray, prob: np.ndarray, n_experts: int, n_shared: int,
                  tile_m: int = 128) -> dict:
    """A dispatch plan (dispatch_plan's arrays plus perm_prob, and the routes'
    idx / prob [N, k]) extended by n_shared shared experts (moe.py:185-198,
    :221-234: every token through each, the sum scaled by 1/sqrt(n_shared))
    as experts E..E+S-1 with probability 1/sqrt(S) for every token, their
    rows after the routed ones: expert E+s holds tokens 0..N-1 at rows
    N*k + s*N + t.  Summing each token's k + S rows, each row scaled by its
    probability, gives routed + sum_s SwiGLU_s(x) / sqrt(S)."""
    idx = np.asarray(idx, dtype=np.int64)
    n, k = idx.shape
    s_ = int(n_shared)
    p = np.float32(1.0 / np.sqrt(float(s_)))
    rows = n * k
    shared_pos = rows + np.arange(s_)[None, :] * n + np.arange(n)[:, None]
    tiles = -(-n // tile_m)
    step = np.arange(1, s_ + 1)
    return dict(
        topk_idx=np.concatenate([idx, np.broadcast_to(n_experts + np.arange(s_), (n, s_))], 1),
        topk_prob=np.concatenate([np.asarray(prob, np.float32), np.full((n, s_), p, np.float32)], 1),
        counts=np.concatenate([plan["counts"], np.full(s_, n)]),
        offsets=np.concatenate([plan["offsets"], plan["offsets"][-1] + n * step]),
        tile_offsets=np.concatenate([plan["tile_offsets"], plan["tile_offsets"][-1] + tiles * step]),
        perm_token=np.concatenate([plan["perm_token"], np.tile(np.arange(n), s_)]),
        perm_prob=np.concatenate([np.asarray(plan["perm_prob"], np.float32),
                                  np.full(n * s_, p, np.float32)]),
        route_pos=np.concatenate([np.asarray(plan["route_pos"]).reshape(n, k), shared_pos],
                                 1).reshape(-1),
    )


def silu(x: np.ndarray) -> np.ndarray:
    return x / (1.0 + np.exp(-x))


def moe_forward(flat: np.ndarray, idx: np.ndarray, prob: np.ndarray, w_gate: np.ndarray,
                w_up: np.ndarray, w_down: np.ndarray, dtype=np.float64) -> np.ndarray:
    """out[t] = sum_s prob[t,s] * W_down[e] (silu(W_gate[e] x_t) * (W_up[e] x_t)), e = idx[t,s].

    moe.py:72-81 computes exactly this (padded bmm, silu(g)*u, bmm, gather,
    probability scale, index_add), in float64 here.
    """
    x = np.asarray(flat, dtype=dtype)
    idx = np.asarray(idx, dtype=np.int64)
    prob = np.asarray(prob, dtype=dtype)
    n, k = idx.shape
    out = np.zeros_like(x)
    for e in np.unique(idx):
        tok, slot = np.nonzero(idx == e)
        xe = x[tok]
        g = xe @ np.asarray(w_gate[e], dtype=dtype).T
        u = xe @ np.asarray(w_up[e], dtype=dtype).T
        y = (silu(g) * u) @ np.asarray(w_down[e], dtype=dtype).T
        np.add.at(out, tok, y * prob[tok, slot][:, None])
    return out


def zipf_expert_bias(n_experts: int, s: float = 1.1, seed: int = 0) -> np.ndarray:
    """Per-expert router bias b_e = log p_{pi(e)}, p_r proportional to r^-s.

    Build-side input of the isolated-MoE workload (the reference router has no
    bias: context_router.py:28).  pi is a seeded permutation of the ranks.
    """
    ranks = np.arange(1, n_experts + 1, dtype=np.float64)
    p = ranks ** (-s)
    p /= p.sum()
    perm = np.random.default_rng(seed).permutation(n_experts)
    return np.log(p[perm]).astype(np.float32)
