"""Host-side plan logic (CPU tensors): a routing plan extended by shared
experts, applied row by row as the expert kernels do, gives the routed MoE plus
the shared experts' sum / sqrt(n) (moe.py:185-198)."""
import numpy as np
import torch

from hybrid_llm_b200 import kernels
from oracle import routing


def _cpu_plan(idx, prob, e, tile_m=128):
    p = routing.dispatch_plan(idx, e, tile_m)
    i32 = lambda a: torch.from_numpy(np.asarray(a)).to(torch.int32)
    flat_prob = prob.reshape(-1)[p["sort_order"]]
    return kernels.RoutePlan(
        topk_idx=torch.from_numpy(idx).to(torch.int64), topk_prob=torch.from_numpy(prob).float(),
        counts=i32(p["counts"]), offsets=i32(p["offsets"]), tile_offsets=i32(p["tile_offsets"]),
        perm_token=i32(p["perm_token"]), perm_prob=torch.from_numpy(flat_prob).float(),
        route_pos=i32(p["route_pos"]), sort_order=None, tile_m=tile_m)


def _swiglu(x, g, u, d):
    return (routing.silu(x @ g.T) * (x @ u.T)) @ d.T


def test_shared_expert_plan_reproduces_routed_plus_shared():
    rng = np.random.default_rng(0)
    n, dm, f, e, k, ns = 37, 16, 24, 8, 2, 3
    x = rng.normal(size=(n, dm))
    idx, prob = routing.router_topk(rng.normal(size=(n, e)).astype(np.float32), k)
    w = [rng.normal(size=s) * 0.3 for s in ((e + ns, f, dm), (e + ns, f, dm), (e + ns, dm, f))]
    plan = kernels.with_shared_experts(_cpu_plan(idx, prob, e), ns)

    rows = n * (k + ns)
    offsets = plan.offsets.numpy()
    assert plan.n_experts == e + ns and offsets[-1] == rows
    assert np.array_equal(plan.counts.numpy()[e:], [n] * ns)
    assert np.array_equal(np.diff(plan.tile_offsets.numpy())[e:], [1] * ns)  # ceil(37 / 128)
    assert np.array_equal(np.sort(plan.route_pos.numpy()), np.arange(rows))
    assert plan.topk_idx.shape == (n, k + ns) and (plan.topk_idx[:, k:] == torch.arange(e, e + ns)).all()

    # the kernels' semantics: row pos = prob * expert(x[token]), combine = sum of a token's rows
    y = np.zeros((rows, dm))
    tok, pp = plan.perm_token.numpy(), plan.perm_prob.numpy()
    for ex in range(e + ns):
        for pos in range(offsets[ex], offsets[ex + 1]):
            y[pos] = pp[pos] * _swiglu(x[tok[pos]], w[0][ex], w[1][ex], w[2][ex])
    got = y[plan.route_pos.numpy()].reshape(n, k + ns, dm).sum(1)

    want = routing.moe_forward(x, idx, prob, w[0][:e], w[1][:e], w[2][:e])
    want = want + sum(_swiglu(x, w[0][e + s], w[1][e + s], w[2][e + s]) for s in range(ns)) / np.sqrt(ns)
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-7)


def test_zero_shared_experts_keep_the_plan():
    rng = np.random.default_rng(1)
    idx, prob = routing.router_topk(rng.normal(size=(5, 4)).astype(np.float32), 2)
    plan = _cpu_plan(idx, prob, 4)
    assert kernels.with_shared_experts(plan, 0) is plan
