"""Next-token sampling (numpy oracle).

Reference: sample_standalone.py:5383-5423 (_sample_next_token) and the inline
copy in sample() (:5596-5636):
  raw_log_probs = log_softmax(logits)
  repetition penalty over set(generated): l > 0 ? l / rep : l * rep
  temp <= 1e-4: argmax (first maximal index)
  else: /temp; top_k > 0 -> topk (value desc); 0 < top_p < 1 -> sort desc,
        softmax, cumsum, remove where the EXCLUSIVE cumulative > top_p
        (first always kept), softmax of the kept values, multinomial.
The multinomial draw is replaced by a deterministic inverse CDF with a
caller-supplied uniform u: the first candidate whose inclusive cumulative
probability exceeds u, in the order the reference hands to multinomial
(value desc / index asc after top-k or top-p, vocabulary order otherwise).
"""
from __future__ import annotations

import numpy as np


def _log_softmax(x):
    m = x.max()
    return x - (m + np.log(np.exp(x - m).sum()))


def inverse_cdf(probs: np.ndarray, u: float) -> int:
    c = np.cumsum(probs)
    hit = np.nonzero(u < c)[0]
    if hit.size:
        return int(hit[0])
    return int(np.nonzero(probs > 0)[0][-1])


def sample_row(logits, generated, *, temp, top_k, top_p, rep, u, blocked=None):
    """Returns (token, raw log-prob of the token, kept probabilities, candidate ids)."""
    x = np.asarray(logits, dtype=np.float64)
    raw_lp = _log_softmax(x)
    w = x.copy()
    if blocked:
        w[list(blocked)] = -np.inf
    if rep != 1.0 and generated:
        seen = np.array(sorted(set(int(g) for g in generated)), dtype=np.int64)
        sv = w[seen]
        w[seen] = np.where(sv > 0, sv / rep, sv * rep)
    if temp <= 1e-4:
        tok = int(np.argmax(w))
        return tok, raw_lp[tok], None, None
    w = w / temp
    v = w.shape[0]
    nucleus = 0.0 < top_p < 1.0
    if top_k > 0 or nucleus:
        # torch.topk / torch.sort order: value desc (ties: index asc)
        order = np.lexsort((np.arange(v), -w))
        cand = order[:min(top_k, v)] if top_k > 0 else order
    else:
        cand = np.arange(v)  # plain softmax over the vocabulary in index order
    vals = w[cand]
    if nucleus:
        p = np.exp(vals - vals.max())
        p /= p.sum()
        cum = np.cumsum(p)
        remove = np.zeros_like(cum, dtype=bool)
        remove[1:] = cum[:-1] > top_p
        vals = np.where(remove, -np.inf, vals)
    p = np.exp(vals - vals.max())
    p /= p.sum()
    i = inverse_cdf(p, u)
    tok = int(cand[i])
    return tok, raw_lp[tok], p, cand


def sample_next_token(logits, generated, *, temp, top_k, top_p, rep, uniforms, blocked=None):
    """Batch version: generated is a list (one per row) of token lists."""
    logits = np.asarray(logits)
    toks, lps = [], []
    for r in range(logits.shape[0]):
        t, lp, _, _ = sample_row(logits[r], generated[r], temp=temp, top_k=top_k, top_p=top_p,
                                 rep=rep, u=float(uniforms[r]), blocked=blocked)
        toks.append(t)
        lps.append(lp)
    return np.array(toks, dtype=np.int64), np.array(lps)
