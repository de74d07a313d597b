"""GPU: router top-k and dispatch plan vs the oracle / reference goldens (bit-exact)."""
import numpy as np
import pytest
import torch

import inputs
from conftest import golden
from oracle import routing

pytestmark = pytest.mark.gpu


def _run_route(logits, k, bias=None, fused=True, dev="cuda"):
    from hybrid_llm_b200 import kernels
    lg = torch.from_numpy(np.ascontiguousarray(logits)).to(dev)
    b = None if bias is None else torch.from_numpy(bias).to(dev)
    if fused:
        plan = kernels.route(lg, k, b, with_sort_order=True)
    else:
        idx, prob = kernels.router_topk(lg, k, b)
        plan = kernels.moe_plan(idx, prob, lg.shape[1], with_sort_order=True)
    torch.cuda.synchronize()
    kernels.check_device_status()
    return {k_: (v.cpu().numpy() if isinstance(v, torch.Tensor) else v) for k_, v in vars(plan).items()}


def _check_plan(got, idx, prob, e):
    ref = routing.dispatch_plan(idx, e, tile_m=got["tile_m"])
    np.testing.assert_array_equal(got["topk_idx"], idx)
    np.testing.assert_allclose(got["topk_prob"], prob, rtol=2e-6, atol=1e-7)
    np.testing.assert_array_equal(got["counts"], ref["counts"])
    np.testing.assert_array_equal(got["offsets"], ref["offsets"])
    np.testing.assert_array_equal(got["tile_offsets"], ref["tile_offsets"])
    np.testing.assert_array_equal(got["sort_order"], ref["sort_order"])
    np.testing.assert_array_equal(got["perm_token"], ref["perm_token"])
    np.testing.assert_array_equal(got["route_pos"], ref["route_pos"])
    k = idx.shape[1]
    np.testing.assert_array_equal(got["perm_prob"], got["topk_prob"].reshape(-1)[ref["sort_order"]])
    assert got["sort_order"].size == idx.size


@pytest.mark.parametrize("tag", list(inputs.ROUTER_CASES))
@pytest.mark.parametrize("fused", [True, False])
def test_router_on_reference_logits(cuda, tag, fused):
    g = golden("router")
    k = inputs.ROUTER_CASES[tag][3]
    e = inputs.ROUTER_CASES[tag][2]
    got = _run_route(g[f"{tag}_logits"], k, fused=fused)
    _check_plan(got, g[f"{tag}_idx"], g[f"{tag}_prob"], e)
    np.testing.assert_array_equal(got["sort_order"], g[f"{tag}_stable_order"])


@pytest.mark.parametrize("n,e,k", [(16384, 32, 4), (4096, 64, 8), (1, 16, 2), (257, 8, 2),
                                   (1000, 256, 32), (300, 5, 5), (64, 64, 8)])
@pytest.mark.parametrize("zipf", [False, True])
def test_router_seeded_shapes(cuda, n, e, k, zipf):
    rng = np.random.default_rng(n * 7 + e)
    logits = rng.normal(0, 0.64, (n, e)).astype(np.float32)
    bias = routing.zipf_expert_bias(e) if zipf else None
    idx, prob = routing.router_topk(logits, k, bias)
    for fused in (True, False):
        got = _run_route(logits, k, bias, fused=fused)
        _check_plan(got, idx, prob, e)


def test_router_zero_tokens(cuda):
    from hybrid_llm_b200 import kernels
    plan = kernels.route(torch.zeros(0, 32, device="cuda"), 4)
    torch.cuda.synchronize()
    assert int(plan.offsets[-1]) == 0 and int(plan.tile_offsets[-1]) == 0


def test_router_ties_lowest_index(cuda):
    logits = np.zeros((3, 40), dtype=np.float32)
    logits[0, [3, 7, 33]] = 1.0
    logits[2, :] = 0.5
    got = _run_route(logits, 3)
    assert got["topk_idx"].tolist() == [[3, 7, 33], [0, 1, 2], [0, 1, 2]]


def test_router_rejects_unsupported(cuda):
    from hybrid_llm_b200 import kernels
    with pytest.raises(RuntimeError, match="not supported"):
        kernels.route(torch.zeros(4, 300, device="cuda"), 2)
    with pytest.raises(RuntimeError, match="invalid argument"):
        kernels.route(torch.zeros(4, 8, device="cuda"), 9)


def test_plan_flags_out_of_range_expert(cuda):
    from hybrid_llm_b200 import kernels
    idx = torch.tensor([[0, 9]], device="cuda")
    prob = torch.full((1, 2), 0.5, device="cuda")
    kernels.moe_plan(idx, prob, 8)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="invalid argument"):
        kernels.check_device_status()
