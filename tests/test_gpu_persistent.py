"""GPU: the batch-1 decode step as one persistent launch (llmyb_decode_persistent).

Checked three ways:
* against the per-sub-layer decode kernels from the same prefilled state
  (teacher-forced tokens; logits within 2e-2 of max |ref|, the experts chosen
  equal except at near ties of the fp32 router logits) on the mini model, and
  the small LLMY model against the fp64 oracle, routing-aware;
* against the reference's own logits (row 0 of the mini golden, which is
  independent of row 1), routing-aware (tests/route_parity.py);
* replayed in a CUDA graph by GreedyDecoder: the same tokens as eager steps.
"""
import numpy as np
import pytest
import torch

import inputs
from conftest import golden

pytestmark = pytest.mark.gpu

STEP_REL = 2e-2


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / np.abs(b).max())


def _model(cfg, sd=None):
    from hybrid_llm_b200.model import LoopedHybridModel
    from hybrid_llm_b200.weights import ModelWeights, synthetic_state_dict
    sd = synthetic_state_dict(cfg, seed=0) if sd is None else sd
    return LoopedHybridModel(ModelWeights.from_state_dict(cfg, sd, "cuda"))


def _compare_paths(m, ids, steps):
    from hybrid_llm_b200 import kernels, persistent
    from hybrid_llm_b200.state import RecurrentState
    assert persistent.supported(m, 1)
    out = m.forward(torch.from_numpy(ids).cuda(), last_logits_only=True)
    saved = out.state.state_dict()
    st_a = RecurrentState(m.cfg, 1, "cuda")
    st_a.load_state_dict(saved)
    st_b = RecurrentState(m.cfg, 1, "cuda")
    st_b.load_state_dict(saved)
    tok = out.logits[:, -1].float().argmax(-1)
    worst = 0.0
    for s in range(steps):
        m.decode_persistent, m.route_log = False, []
        a = m.decode_step(tok, st_a).float().cpu().numpy()
        ra = torch.cat(m.route_log).cpu().numpy()
        m.decode_persistent, m.route_log = True, []
        b = m.decode_step(tok, st_b).float().cpu().numpy()
        rb = torch.cat(m.route_log).cpu().numpy()
        m.route_log = None
        assert int(st_b.positions[0]) == int(st_a.positions[0])
        e = _rel(b, a)
        worst = max(worst, e)
        assert e < STEP_REL, (s, e)
        assert ra.shape == rb.shape
        flips = (np.sort(ra, -1) != np.sort(rb, -1)).any(-1).sum()
        assert flips <= 1, (s, flips)   # a near tie may break the other way once
        tok = torch.from_numpy(a.argmax(-1)).cuda()
    kernels.check_device_status()
    return worst


def test_persistent_matches_kernel_chain_mini(cuda):
    m = _model(inputs.mini_config())
    print("mini worst", _compare_paths(m, inputs.mini_prompt()[:1], 8))


def test_persistent_small_llmy_vs_oracle(cuda):
    """The small LLMY model at full width (200-token prompt, 6 teacher-forced
    decode steps) against the fp64 oracle forced onto the GPU's expert choices
    (tests/route_parity.py): path against path is not meaningful here because
    one near tie of the router logits may resolve differently between two fp32
    summation orders and move the logits by ~20 %."""
    import route_parity
    from hybrid_llm_b200.config import small_llmy_config
    from hybrid_llm_b200.weights import synthetic_state_dict
    from oracle.model import OracleModel
    cfg = small_llmy_config()
    sd = synthetic_state_dict(cfg, seed=0)
    m = _model(cfg, sd)
    orc = OracleModel(cfg, sd)
    rng = np.random.default_rng(3)
    ids = rng.integers(0, cfg.vocab_size, size=(1, 200)).astype(np.int64)
    toks = rng.integers(0, cfg.vocab_size, size=(1, 6)).astype(np.int64)
    stats = route_parity.check_model(m, orc, ids, toks)
    print("small LLMY", stats)


def test_persistent_matches_reference_golden(cuda):
    import route_parity
    from hybrid_llm_b200.weights import synthetic_state_dict
    from oracle.model import OracleModel
    g = golden("model")
    cfg = inputs.mini_config()
    sd = synthetic_state_dict(cfg, seed=0)
    m = _model(cfg, sd)
    orc = OracleModel(cfg, {k: sd[k] for k in sd})
    stats = route_parity.check_model(m, orc, inputs.mini_prompt()[:1], g["mini_tokens"][:1],
                                     g["mini_prefill_last"][:1], g["mini_step_logits"][:1])
    print("golden", stats)
    assert stats["golden_compared"] >= 1


def test_persistent_graph_replay_matches_eager(cuda):
    from hybrid_llm_b200.model import GreedyDecoder
    m = _model(inputs.mini_config())
    ids = torch.from_numpy(inputs.mini_prompt()[:1]).cuda()
    toks = []
    for use_graph in (False, True):
        o = m.forward(ids, last_logits_only=True)
        dec = GreedyDecoder(m, o.state, use_graph=use_graph)
        dec.prime(o.logits[:, -1].float().argmax(-1))
        toks.append(torch.stack([dec.step().clone() for _ in range(10)], 1).cpu())
    assert torch.equal(toks[0], toks[1])


def test_fused_greedy_matches_the_sampler(cuda):
    """The LM head fused with greedy sampling (first maximal logit, its raw
    log-softmax, its bit in the seen mask) against the same persistent step's
    logits handed to the sampler kernel (temperature 0): identical tokens and
    masks, log-probabilities within 1e-5."""
    from hybrid_llm_b200 import kernels
    from hybrid_llm_b200.state import RecurrentState
    from hybrid_llm_b200.config import small_llmy_config
    for cfg, t in ((inputs.mini_config(), 50), (small_llmy_config(), 64)):
        m = _model(cfg)
        assert m.greedy_fused(1)
        ids = torch.from_numpy(np.random.default_rng(1).integers(0, cfg.vocab_size, (1, t))).cuda()
        out = m.forward(ids, last_logits_only=True)
        sts = []
        for _ in range(2):
            st = RecurrentState(cfg, 1, "cuda")
            st.load_state_dict(out.state.state_dict())
            sts.append(st)
        words = (cfg.vocab_size + 31) // 32
        seen = [torch.zeros(1, words, dtype=torch.int32, device="cuda") for _ in range(2)]
        tok_a = out.logits[:, -1].float().argmax(-1)
        tok_b = tok_a.clone()
        lp_b = torch.zeros(1, device="cuda")
        for _ in range(12):
            logits = m.decode_step(tok_a, sts[0])
            tok_a, lp_a = kernels.sample(logits, temperature=0.0, top_k=0, top_p=1.0,
                                         seen=seen[0], update_seen=True)
            m.decode_step_greedy(tok_b, sts[1], tok_b, lp_b, seen[1].view(-1))
            torch.cuda.synchronize()
            assert torch.equal(tok_a, tok_b)
            assert abs(float(lp_a) - float(lp_b)) < 1e-5, (float(lp_a), float(lp_b))
            assert torch.equal(seen[0], seen[1])
        kernels.check_device_status()
