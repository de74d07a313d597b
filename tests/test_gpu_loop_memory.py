"""GPU: the loop memory between recurrent loops (model/loop_memory.py:36-66,
LatentAttention mla_memory.py:66-86; model/model.py:608-667 prefill,
:840-891 decode).

The three per-token kernels against numpy (fp32 tolerance), the mini model
with three loops against the reference's own outputs (tests/golden/
loop_mem.npz: prefill and four greedy decode steps) at the bf16 logit
tolerance, and the same hook on four hyper-connection streams against the
fp64 oracle.
"""
import dataclasses

import numpy as np
import pytest
import torch

import inputs
from conftest import golden

pytestmark = pytest.mark.gpu

LOGIT_REL = 3e-2    # max |logits - ref| / max |ref|


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.abs(a - b).max() / np.abs(b).max()


@pytest.mark.parametrize("n,s,w", [(5, 1, 256), (70, 4, 768), (3, 2, 2048)])
def test_loop_mem_norm(cuda, n, s, w):
    from hybrid_llm_b200 import kernels
    rng = np.random.default_rng(n)
    x = rng.normal(1.0, 2.0, (n, s * w)).astype(np.float32)
    lw, lb = rng.normal(1, 0.1, w).astype(np.float32), rng.normal(0, 0.1, w).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    mean = kernels.loop_mem_norm(xt, s, w).cpu().numpy()
    ln = kernels.loop_mem_norm(xt, s, w, torch.from_numpy(lw).cuda(),
                               torch.from_numpy(lb).cuda()).cpu().numpy()
    m = x.astype(np.float64).reshape(n, s, w).mean(1)
    want = (m - m.mean(-1, keepdims=True)) / np.sqrt(m.var(-1, keepdims=True) + 1e-5) * lw + lb
    assert _rel(mean, m) < 1e-6 and _rel(ln, want) < 1e-5


@pytest.mark.parametrize("n,j,h,hd", [(7, 1, 4, 32), (33, 2, 4, 32), (5, 5, 3, 80)])
def test_loop_mem_attend_and_add(cuda, n, j, h, hd):
    from hybrid_llm_b200 import kernels
    rng = np.random.default_rng(j)
    q = rng.normal(size=(n, h * hd)).astype(np.float32)
    kv = rng.normal(size=(j, n, 2 * h * hd)).astype(np.float32)
    got = kernels.loop_mem_attend(torch.from_numpy(q).cuda(), torch.from_numpy(kv).cuda(), j, h,
                                  hd).cpu().numpy()
    k = kv[..., :h * hd].reshape(j, n, h, hd).astype(np.float64)
    v = kv[..., h * hd:].reshape(j, n, h, hd).astype(np.float64)
    sc = np.einsum("nhd,jnhd->nhj", q.reshape(n, h, hd), k) / np.sqrt(hd)
    p = np.exp(sc - sc.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    want = np.einsum("nhj,jnhd->nhd", p, v).reshape(n, -1)
    assert _rel(got, want) < 1e-5
    s, d = 2, 64
    streams = torch.from_numpy(rng.normal(size=(n, s * d)).astype(np.float32)).cuda()
    delta = torch.from_numpy(rng.normal(size=(n, d)).astype(np.float32)).cuda()
    before = streams.clone()
    kernels.loop_mem_add(streams, s, delta, 0.37)
    want = before.view(n, s, d) + 0.37 * delta[:, None]
    assert torch.allclose(streams.view(n, s, d), want, rtol=1e-6, atol=1e-6)


def _model(cfg):
    from hybrid_llm_b200.model import LoopedHybridModel
    from hybrid_llm_b200.weights import ModelWeights, synthetic_state_dict
    return LoopedHybridModel(ModelWeights.from_state_dict(cfg, synthetic_state_dict(cfg, seed=0),
                                                          "cuda"))


@pytest.mark.parametrize("fused", [True, False])
def test_loop_memory_model_prefill_and_greedy_decode(cuda, fused):
    g = golden("loop_mem")
    m = _model(inputs.loop_memory_config())
    m.decode_fused = fused
    ids = torch.from_numpy(inputs.mini_prompt()).cuda()
    out = m.forward(ids, last_logits_only=True)
    lg = out.logits[:, -1].float().cpu().numpy()
    assert _rel(lg, g["lm_prefill_last"]) < LOGIT_REL, _rel(lg, g["lm_prefill_last"])
    state = out.state
    tok = torch.from_numpy(g["lm_tokens"][:, 0]).cuda()
    tol = LOGIT_REL * np.abs(g["lm_prefill_last"]).max()
    for i in range(g["lm_tokens"].shape[1]):
        lg = m.decode_step(tok, state).float().cpu().numpy()
        ref = g["lm_step_logits"][:, i]
        assert _rel(lg, ref) < LOGIT_REL, (i, _rel(lg, ref))
        if i + 1 < g["lm_tokens"].shape[1]:
            want = g["lm_tokens"][:, i + 1]
            for r in np.nonzero(lg.argmax(-1) != want)[0]:
                top2 = np.sort(ref[r])[-2:]
                assert top2[1] - top2[0] <= tol, (i, r)
            tok = torch.from_numpy(want).cuda()  # teacher-force the reference


def test_loop_memory_with_hyper_connections_vs_oracle(cuda):
    """Four mHC streams: the hook reads the stream mean and adds to every
    stream (loop_memory.py:45, :50-52); prefill and two decode steps against
    the fp64 oracle (pinned to the reference for both features)."""
    from hybrid_llm_b200.weights import synthetic_state_dict
    from oracle.model import OracleModel
    cfg = dataclasses.replace(inputs.loop_memory_config(), mhc_streams=4, mhc_iterations=10)
    m = _model(cfg)
    sd = synthetic_state_dict(cfg, seed=0)
    orc = OracleModel(cfg, {k: sd[k] for k in sd})
    ids = inputs.mini_prompt()
    out = m.forward(torch.from_numpy(ids).cuda(), last_logits_only=True)
    ref, st = orc.forward(ids)
    assert _rel(out.logits[:, -1].float().cpu().numpy(), ref[:, -1]) < LOGIT_REL
    tok = ref[:, -1].argmax(-1)
    state = out.state
    for _ in range(2):
        got = m.decode_step(torch.from_numpy(tok).cuda(), state).float().cpu().numpy()
        ref_s, st = orc.decode_step(tok, st)
        assert _rel(got, ref_s) < LOGIT_REL, _rel(got, ref_s)
        tok = ref_s.argmax(-1)
