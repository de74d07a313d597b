"""GPU: the CSA remote compressed branch (model/layers/csa.py:77-131 prefill,
:208-256 decode; compressed_attention.py:85-206).

The prefill and decode kernels against the oracle's compressor (bf16
tolerance) and its top-k summary attention over the same bf16 summaries;
the mini model with the branch on against the reference's own outputs
(tests/golden/csa_remote.npz: 4-token summaries, top-3, prefill and eight
teacher-forced decode steps), and mHC + router context + remote branch +
shared experts together (tests/golden/combined.npz), both routing-aware
(tests/route_parity.py): one of those decode steps has a top-2 / top-3
router margin of 0.24 % of the logit range, which the bf16 path may resolve
the other way.
"""
import numpy as np
import pytest
import torch

import inputs
from conftest import golden

pytestmark = pytest.mark.gpu

LOGIT_REL = 3e-2    # max |logits - ref| / max |ref|
BF16_REL = 2e-2     # bf16 storage, fp32 arithmetic


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


def _bf(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16)


def _f64(t):
    return t.float().cpu().numpy().astype(np.float64)


def _visible_summaries(mem):
    """The oracle memory's visible entries (decode appends invisible ones)."""
    keep = mem["pos"][0] >= 0
    return mem["keys"][:, keep], mem["values"][:, keep], mem["pos"][:, keep]


@pytest.mark.parametrize("b,t,d,h,dh,ratio,top_k", [
    (1, 50, 64, 2, 32, 4, 3), (2, 130, 128, 4, 32, 4, 32), (1, 3, 64, 2, 32, 4, 3),
    (2, 257, 256, 8, 64, 8, 16)])
def test_remote_prefill_matches_oracle(cuda, b, t, d, h, dh, ratio, top_k):
    """The compressor's summaries against the oracle's (bf16 tolerance), then
    the top-k attention on those same bf16 summaries against the oracle's
    (identical selections up to fp32 summation order)."""
    from hybrid_llm_b200 import kernels
    from oracle import attention
    rng = np.random.default_rng(t + d)
    x = _bf(rng.normal(size=(b, t, d)))
    q = _bf(rng.normal(size=(b, t, h * dh)))
    wk = _bf(rng.normal(0, 0.3, (h * dh, d)))
    wv = _bf(rng.normal(0, 0.3, (d, d)))
    w_comp = torch.cat([wk, wv]).cuda()
    pend_sum = torch.empty(b, d, device="cuda")
    pend_cnt = torch.empty(b, dtype=torch.int32, device="cuda")
    remote, summ = kernels.csa_remote_prefill(x.cuda(), q.cuda(), w_comp, ratio, top_k, h,
                                              pend_sum, pend_cnt)
    torch.cuda.synchronize()
    mem = attention.compress_prefill(_f64(x), _f64(wk), _f64(wv), ratio)
    n = t // ratio
    assert summ.shape[1] == n
    if n:
        assert _rel(_f64(summ[..., :h * dh]), mem["keys"]) < BF16_REL
        assert _rel(_f64(summ[..., h * dh:]), mem["values"]) < BF16_REL
    np.testing.assert_allclose(pend_sum.cpu().numpy(), mem["sum"], rtol=1e-5, atol=1e-4)
    np.testing.assert_array_equal(pend_cnt.cpu().numpy(), mem["count"])
    want = attention.remote_attention(_f64(q).reshape(b, t, h, dh), _f64(summ[..., :h * dh]),
                                      _f64(summ[..., h * dh:]), mem["pos"], np.arange(t), top_k)
    if np.abs(want).max() == 0:
        assert float(remote.abs().max()) == 0
    else:
        assert _rel(_f64(remote), want) < BF16_REL, _rel(_f64(remote), want)


def test_remote_decode_steps_match_oracle(cuda):
    """A prompt of 10 tokens (two summaries + two pending), then 13 decode
    steps (three more blocks complete), B = 3: at every step the stored
    summaries against the oracle's compress_step (bf16 tolerance), and the
    remote attention over those stored bf16 summaries against the oracle's."""
    from hybrid_llm_b200 import kernels
    from oracle import attention
    b, t, d, h, dh, ratio, top_k, steps = 3, 10, 128, 4, 32, 4, 3, 13
    rng = np.random.default_rng(11)
    x = _bf(rng.normal(size=(b, t + steps, d)))
    q = _bf(rng.normal(size=(b, t + steps, h * dh)))
    wk, wv = _bf(rng.normal(0, 0.3, (h * dh, d))), _bf(rng.normal(0, 0.3, (d, d)))
    w_comp = torch.cat([wk, wv]).cuda()
    cap = 8
    mem_k = torch.zeros(b, cap, h * dh, dtype=torch.bfloat16, device="cuda")
    mem_v = torch.zeros(b, cap, d, dtype=torch.bfloat16, device="cuda")
    count = torch.zeros(b, dtype=torch.int32, device="cuda")
    pend_sum = torch.zeros(b, d, device="cuda")
    pend_cnt = torch.zeros(b, dtype=torch.int32, device="cuda")
    xc, qc = x.cuda(), q.cuda()
    _, summ = kernels.csa_remote_prefill(xc[:, :t].contiguous(), qc[:, :t].contiguous(), w_comp,
                                         ratio, top_k, h, pend_sum, pend_cnt)
    n = summ.shape[1]
    mem_k[:, :n] = summ[..., :h * dh]
    mem_v[:, :n] = summ[..., h * dh:]
    count.fill_(n)
    mem = attention.compress_prefill(_f64(x[:, :t]), _f64(wk), _f64(wv), ratio)
    out = torch.empty(b, 2 * d, dtype=torch.bfloat16, device="cuda")
    for s in range(steps):
        pos = t + s
        kernels.csa_remote_step(xc[:, pos].contiguous(), qc[:, pos].contiguous(), w_comp, ratio,
                                top_k, h, mem_k, mem_v, count, pend_sum, pend_cnt, out[:, d:])
        torch.cuda.synchronize()
        mem = attention.compress_step(mem, _f64(x[:, pos]), _f64(wk), _f64(wv), ratio, pos)
        keys, values, kpos = _visible_summaries(mem)
        cnt = int(count[0])
        assert (count.cpu().numpy() == keys.shape[1]).all()
        np.testing.assert_array_equal(pend_cnt.cpu().numpy(), mem["count"])
        assert _rel(_f64(mem_k[:, :cnt]), keys) < BF16_REL
        assert _rel(_f64(mem_v[:, :cnt]), values) < BF16_REL
        want = attention.remote_attention(_f64(q[:, pos]).reshape(b, 1, h, dh),
                                          _f64(mem_k[:, :cnt]), _f64(mem_v[:, :cnt]), kpos,
                                          np.array([pos]), top_k)[:, 0]
        assert _rel(_f64(out[:, d:]), want) < BF16_REL, (s, _rel(_f64(out[:, d:]), want))
    kernels.check_device_status()


def _model_and_oracle(cfg):
    from hybrid_llm_b200.model import LoopedHybridModel
    from hybrid_llm_b200.weights import ModelWeights, synthetic_state_dict
    from oracle.model import OracleModel
    sd = synthetic_state_dict(cfg, seed=0)
    m = LoopedHybridModel(ModelWeights.from_state_dict(cfg, sd, "cuda"))
    return m, OracleModel(cfg, {k: sd[k] for k in sd})


def _golden_run(cfg, g, tag, fused=True):
    """Prefill and the golden's teacher-forced decode steps, routing-aware
    (route_parity): against the oracle with the GPU's expert choices, and
    against the reference's logits wherever routing agreed."""
    import route_parity
    m, orc = _model_and_oracle(cfg)
    m.decode_fused = fused
    stats = route_parity.check_model(m, orc, inputs.mini_prompt(), g[f"{tag}_tokens"],
                                     g[f"{tag}_prefill_last"], g[f"{tag}_step_logits"],
                                     logit_rel=LOGIT_REL)
    print(tag, stats)
    assert stats["golden_compared"] >= 1


@pytest.mark.parametrize("fused", [True, False])
def test_csa_remote_model_prefill_and_greedy_decode(cuda, fused):
    _golden_run(inputs.csa_remote_config(), golden("csa_remote"), "cr", fused)


def test_combined_features_model_prefill_and_greedy_decode(cuda):
    """Hyper-connections (4 streams), the router's local context, the CSA remote
    branch and shared experts together (the reference's default feature set)."""
    _golden_run(inputs.combined_config(), golden("combined"), "cb")
