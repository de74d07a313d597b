"""Expert-parallel dispatch / combine (numpy oracle) — TEST INFRASTRUCTURE.

The reference runs the routed experts of model/layers/moe.py:29-82 on one
device; expert parallelism deploys the same math over W ranks, rank q owning
experts [q*El, (q+1)*El).  This module restates, on the exact wire format of
hybrid_llm_b200/csrc/ep.cu, what each step must produce, so that the CUDA
kernels (GPU tests) and the host-side exchange (gloo tests) can be checked:

  dispatch segment for peer q (bf16 rows of D elements, uint16 bit patterns):
    rows [0, H): int32 counts[El] then fp32 probs[C]   (header)
    rows [H, H+C): the routed token rows of the local plan range
                   [offsets[q*El], offsets[(q+1)*El]) in plan order
  return segment: C rows, the expert outputs in dispatch row order.

Buffers here are numpy uint16 arrays holding bf16 bit patterns.
"""
from __future__ import annotations

import numpy as np

from .routing import silu


def header_rows(el: int, capacity: int, d: int) -> int:
    return -(-4 * (el + capacity) // (2 * d))


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float values to bf16 (nearest even); returns uint16 bit patterns."""
    f = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = f + np.uint32(0x7FFF) + ((f >> np.uint32(16)) & np.uint32(1))
    return (rounded >> np.uint32(16)).astype(np.uint16)


def bf16_value(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def dispatch_pack(x_bits: np.ndarray, offsets, perm_token, perm_prob, route_pos, n_experts: int,
                  world: int, capacity: int, send: np.ndarray, ret_route_pos: np.ndarray) -> None:
    """Fill send [W, H+C, D] (uint16) and ret_route_pos [n_routes] in place."""
    el = n_experts // world
    d = x_bits.shape[1]
    h = header_rows(el, capacity, d)
    offsets = np.asarray(offsets, dtype=np.int64)
    for q in range(world):
        b, e = offsets[q * el], offsets[(q + 1) * el]
        cnt = e - b
        send[q, h:h + cnt] = x_bits[np.asarray(perm_token[b:e], dtype=np.int64)]
        hdr = send[q, :h].reshape(-1).view(np.int32)
        hdr[:el] = np.diff(offsets[q * el:(q + 1) * el + 1])
        hdr.view(np.float32)[el:el + cnt] = np.asarray(perm_prob[b:e], dtype=np.float32)
    pos = np.asarray(route_pos, dtype=np.int64)
    expert = np.searchsorted(offsets, pos, side="right") - 1
    q = expert // el
    ret_route_pos[:] = q * capacity + (pos - offsets[q * el])


def recv_plan(recv: np.ndarray, world: int, capacity: int, el: int):
    """Local plan over received segments recv [W, H+C, D] (uint16).

    Returns offsets_l [El+1], perm_token_l, perm_prob_l, out_row (length
    offsets_l[El]); rows of an expert ordered by (source rank, source order).
    """
    d = recv.shape[2]
    h = header_rows(el, capacity, d)
    counts = np.stack([recv[p, :h].reshape(-1).view(np.int32)[:el] for p in range(world)])
    probs = [recv[p, :h].reshape(-1).view(np.int32).view(np.float32)[el:el + capacity]
             for p in range(world)]
    offsets_l = np.concatenate([[0], np.cumsum(counts.sum(0))]).astype(np.int64)
    perm_token, perm_prob, out_row = [], [], []
    for e in range(el):
        for p in range(world):
            base = counts[p, :e].sum()
            for j in range(counts[p, e]):
                i = base + j
                perm_token.append(p * (h + capacity) + h + i)
                perm_prob.append(probs[p][i])
                out_row.append(p * capacity + i)
    return (offsets_l, np.asarray(perm_token, dtype=np.int64),
            np.asarray(perm_prob, dtype=np.float32), np.asarray(out_row, dtype=np.int64))


def expert_rows(x_rows: np.ndarray, prob: np.ndarray, w13_gate: np.ndarray, w13_up: np.ndarray,
                w_down: np.ndarray) -> np.ndarray:
    """p * W_down (silu(W_gate x) * (W_up x)) for rows of ONE expert, with the
    kernels' rounding points: h rounded to bf16, output rounded to bf16
    (moe.py:72-81).  Float64 arithmetic; returns uint16 bit patterns."""
    x = x_rows.astype(np.float64)
    g = x @ w13_gate.astype(np.float64).T
    u = x @ w13_up.astype(np.float64).T
    hb = bf16_value(bf16_bits(silu(g) * u)).astype(np.float64)
    y = (hb @ w_down.astype(np.float64).T) * prob.astype(np.float64)[:, None]
    return bf16_bits(y)


def experts_to(recv: np.ndarray, offsets_l, perm_token_l, perm_prob_l, out_row, w_gate, w_up,
               w_down, y_out: np.ndarray) -> None:
    """y_out[out_row[pos]] = expert outputs of the local plan (uint16 rows).
    w_gate / w_up / w_down: the rank's local experts [El, F, D] / [El, D, F]."""
    rows = recv.reshape(-1, recv.shape[-1])
    for e in range(len(offsets_l) - 1):
        a, b = int(offsets_l[e]), int(offsets_l[e + 1])
        if b == a:
            continue
        xr = bf16_value(rows[np.asarray(perm_token_l[a:b], dtype=np.int64)])
        y_out[np.asarray(out_row[a:b], dtype=np.int64)] = expert_rows(
            xr, np.asarray(perm_prob_l[a:b]), w_gate[e], w_up[e], w_down[e])


def combine(y_rows: np.ndarray, route_pos, n_tokens: int, k: int) -> np.ndarray:
    """out[t] = sum_s y_rows[route_pos[t*k+s]] in fp32, slot order (the sum of
    llmyb_add_rmsnorm_routed)."""
    pos = np.asarray(route_pos, dtype=np.int64).reshape(n_tokens, k)
    vals = bf16_value(y_rows[pos])  # [N, k, D]
    out = np.zeros((n_tokens, y_rows.shape[1]), dtype=np.float32)
    for s in range(k):
        out += vals[:, s]
    return out
