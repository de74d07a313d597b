"""Host-side plan logic: a routing plan extended by shared experts
(oracle.routing.append_shared, the restatement the llmyb_plan_append_shared
kernel is checked against bit for bit on the GPU), applied row by row as the
expert kernels do, gives the routed MoE plus the shared experts' sum /
sqrt(n) (moe.py:185-198)."""
import numpy as np
import pytest

from oracle import routing


def _plan(idx, prob, e, tile_m=128):
    p = routing.dispatch_plan(idx, e, tile_m)
    p["perm_prob"] = prob.reshape(-1)[p["sort_order"]].astype(np.float32)
    return p


def _swiglu(x, g, u, d):
    return (routing.silu(x @ g.T) * (x @ u.T)) @ d.T


@pytest.mark.parametrize("n,e,k,ns,tile_m", [(37, 8, 2, 3, 128), (300, 16, 4, 1, 128),
                                             (5, 4, 2, 2, 256)])
def test_shared_expert_plan_reproduces_routed_plus_shared(n, e, k, ns, tile_m):
    rng = np.random.default_rng(n)
    dm, f = 16, 24
    x = rng.normal(size=(n, dm))
    idx, prob = routing.router_topk(rng.normal(size=(n, e)).astype(np.float32), k)
    w = [rng.normal(size=s) * 0.3 for s in ((e + ns, f, dm), (e + ns, f, dm), (e + ns, dm, f))]
    plan = routing.append_shared(_plan(idx, prob, e, tile_m), idx, prob, e, ns, tile_m)

    rows = n * (k + ns)
    offsets = plan["offsets"]
    assert len(plan["counts"]) == e + ns and offsets[-1] == rows
    assert np.array_equal(plan["counts"][e:], [n] * ns)
    assert np.array_equal(np.diff(plan["tile_offsets"])[e:], [-(-n // tile_m)] * ns)
    assert np.array_equal(np.sort(plan["route_pos"]), np.arange(rows))
    assert plan["topk_idx"].shape == (n, k + ns)
    assert (plan["topk_idx"][:, k:] == np.arange(e, e + ns)).all()

    # the kernels' semantics: row pos = prob * expert(x[token]), combine = sum of a token's rows
    y = np.zeros((rows, dm))
    tok, pp = plan["perm_token"], plan["perm_prob"]
    for ex in range(e + ns):
        for pos in range(offsets[ex], offsets[ex + 1]):
            y[pos] = pp[pos] * _swiglu(x[tok[pos]], w[0][ex], w[1][ex], w[2][ex])
    got = y[plan["route_pos"]].reshape(n, k + ns, dm).sum(1)

    want = routing.moe_forward(x, idx, prob, w[0][:e], w[1][:e], w[2][:e])
    want = want + sum(_swiglu(x, w[0][e + s], w[1][e + s], w[2][e + s]) for s in range(ns)) / np.sqrt(ns)
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-7)
