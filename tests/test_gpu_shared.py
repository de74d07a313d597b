"""GPU: shared experts (model/layers/moe.py:185-198 prefill, :221-234 decode).

The plan extension kernel against its restatement (oracle.routing.append_shared)
bit for bit; the routed + shared expert output of one MoE call against the
fp64 oracle; and the mini model with two shared experts against the
reference's own outputs (tests/golden/shared.npz: prefill and four greedy
decode steps), at the bf16 logit tolerance.
"""
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


@pytest.mark.parametrize("n,e,k,ns,tile_m", [(37, 8, 2, 3, 128), (1, 16, 2, 4, 128),
                                             (2048, 32, 4, 2, 256), (0, 8, 2, 1, 128)])
def test_plan_append_shared_matches_oracle(cuda, n, e, k, ns, tile_m):
    from hybrid_llm_b200 import kernels
    from oracle import routing
    rng = np.random.default_rng(n + ns)
    logits = rng.normal(size=(n, e)).astype(np.float32)
    plan = kernels.route(torch.from_numpy(logits).cuda(), k, tile_m=tile_m)
    got = kernels.plan_append_shared(plan, ns)
    torch.cuda.synchronize()
    idx, prob = plan.topk_idx.cpu().numpy(), plan.topk_prob.cpu().numpy()
    base = {f: getattr(plan, f).cpu().numpy() for f in
            ("counts", "offsets", "tile_offsets", "perm_token", "perm_prob", "route_pos")}
    want = routing.append_shared(base, idx, prob, e, ns, tile_m)
    for f, ref in want.items():
        np.testing.assert_array_equal(getattr(got, f).cpu().numpy().reshape(ref.shape), ref,
                                      err_msg=f)


@pytest.mark.parametrize("n,path", [(3, "decode"), (700, "grouped")])
def test_routed_plus_shared_experts_match_oracle(cuda, n, path):
    """One MoE call with S = 2 shared experts: the expert kernels over the
    extended plan and the routed combine, against the oracle's SparseMoE
    (routed experts + sum of shared SwiGLU / sqrt(S)); bf16 tolerance 2e-2."""
    from hybrid_llm_b200 import kernels
    from oracle import routing
    d, e, k, f, ns = 256, 8, 2, 256, 2
    rng = np.random.default_rng(n)
    bf = lambda a: torch.from_numpy(np.asarray(a, np.float32)).to(torch.bfloat16)
    x = bf(rng.normal(size=(n, d)))
    logits = rng.normal(size=(n, e)).astype(np.float32)
    wg, wu = bf(rng.normal(0, 0.05, (e + ns, f, d))), bf(rng.normal(0, 0.05, (e + ns, f, d)))
    wd = bf(rng.normal(0, 0.05, (e + ns, d, f)))
    plan = kernels.plan_append_shared(kernels.route(torch.from_numpy(logits).cuda(), k,
                                                    tile_m=128), ns)
    y = kernels.moe_experts_rows(x.cuda(), plan, kernels.pack_w13(wg.cuda(), wu.cuda()),
                                 wd.cuda(), path=path)
    streams = torch.zeros(n, d, device="cuda")
    kernels.add_rmsnorm_routed(streams, y, plan, None, 1e-6, normalize=False)
    torch.cuda.synchronize()
    f64 = lambda t: t.float().numpy().astype(np.float64)
    idx, prob = routing.router_topk(logits, k)
    ref = routing.moe_forward(f64(x), idx, prob, f64(wg)[:e], f64(wu)[:e], f64(wd)[:e])
    for s in range(ns):
        g = f64(x) @ f64(wg)[e + s].T
        u = f64(x) @ f64(wu)[e + s].T
        ref = ref + (routing.silu(g) * u) @ f64(wd)[e + s].T / np.sqrt(ns)
    assert _rel(streams.cpu().numpy(), ref) < 2e-2, _rel(streams.cpu().numpy(), ref)


def test_shared_experts_model_prefill_and_greedy_decode(cuda):
    from hybrid_llm_b200.model import LoopedHybridModel
    from hybrid_llm_b200.weights import ModelWeights, synthetic_state_dict
    g = golden("shared")
    cfg = inputs.shared_experts_config()
    m = LoopedHybridModel(ModelWeights.from_state_dict(cfg, synthetic_state_dict(cfg, seed=0),
                                                       "cuda"))
    ids = torch.from_numpy(inputs.mini_prompt()).cuda()
    out = m.forward(ids, last_logits_only=True)
    lg = out.logits[:, -1].float().cpu().numpy()
    assert _rel(lg, g["sh_prefill_last"]) < LOGIT_REL, _rel(lg, g["sh_prefill_last"])
    state = out.state
    tok = torch.from_numpy(g["sh_tokens"][:, 0]).cuda()
    tol = LOGIT_REL * np.abs(g["sh_prefill_last"]).max()
    for i in range(g["sh_tokens"].shape[1]):
        lg = m.decode_step(tok, state).float().cpu().numpy()
        ref = g["sh_step_logits"][:, i]
        assert _rel(lg, ref) < LOGIT_REL, (i, _rel(lg, ref))
        if i + 1 < g["sh_tokens"].shape[1]:
            want = g["sh_tokens"][:, i + 1]
            for r in np.nonzero(lg.argmax(-1) != want)[0]:
                top2 = np.sort(ref[r])[-2:]
                assert top2[1] - top2[0] <= tol, (i, r)
            tok = torch.from_numpy(want).cuda()  # teacher-force the reference
