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


# ----------------------------------------------------------------------------
# The reference engine's host sampler, llmy_sample (llmy_cuda/src/llmy.cpp:132-202).
# Single-precision arithmetic in the reference's order (sequential float sums),
# xorshift64 state (13, 7, 17) and u = (state >> 11) / 2^53.  The reference
# orders equal logits by std::partial_sort, which leaves their order open; this
# restatement (and the build) put the lower index first.
_M64 = (1 << 64) - 1


def xorshift64(state: int) -> int:
    state ^= (state << 13) & _M64
    state ^= state >> 7
    state ^= (state << 17) & _M64
    return state & _M64


def engine_host_sample(logits, temperature: float, top_k: int, top_p: float,
                       repetition_penalty: float, recent, rng_state: int):
    """Returns (token, rng_state after the call)."""
    f32 = np.float32
    work = np.array(logits, dtype=np.float32).reshape(-1)
    vocab = work.size
    if vocab <= 0:
        return 0, rng_state
    if top_k <= 0 or top_k > vocab:
        top_k = vocab
    top_k = min(top_k, 256)
    rep = f32(repetition_penalty)
    if rep != f32(1.0) and len(recent) > 0:
        for r in recent:                      # every occurrence applies again
            r = int(r)
            if 0 <= r < vocab:
                v = work[r]
                work[r] = v / rep if v > f32(0.0) else v * rep
    order = np.lexsort((np.arange(vocab), -work))[:top_k]
    temperature = f32(temperature)
    if not (temperature > f32(0.0)):
        return int(order[0]), rng_state
    maxv = work[order[0]]
    probs = np.empty(top_k, dtype=np.float32)
    total = f32(0.0)
    for i in range(top_k):
        z = f32(f32(work[order[i]] - maxv) / temperature)
        e = f32(np.exp(np.float64(z)))         # correctly rounded single-precision exp
        probs[i] = e
        total = f32(total + e)
    for i in range(top_k):
        probs[i] = f32(probs[i] / total)
    cutoff = top_k
    top_p = f32(top_p)
    if f32(0.0) < top_p < f32(1.0):
        cdf = f32(0.0)
        for i in range(top_k):
            cdf = f32(cdf + probs[i])
            if cdf >= top_p:
                cutoff = i + 1
                break
    renorm = f32(0.0)
    for i in range(cutoff):
        renorm = f32(renorm + probs[i])
    for i in range(cutoff):
        probs[i] = f32(probs[i] / renorm)
    rng_state = xorshift64(int(rng_state))
    u = float(rng_state >> 11) / float(1 << 53)
    acc = f32(0.0)
    chosen = int(order[cutoff - 1])
    for i in range(cutoff):
        acc = f32(acc + probs[i])
        if u < float(acc):
            chosen = int(order[i])
            break
    return chosen, rng_state
