"""CPU: the routing/MoE oracle against the reference's golden outputs."""
import numpy as np
import pytest

import inputs
from conftest import golden
from oracle import routing


@pytest.mark.parametrize("tag", list(inputs.ROUTER_CASES))
def test_router_topk_matches_reference(tag):
    g = golden("router")
    c = inputs.router_case(tag)
    assert g[f"{tag}_checksum"] == inputs.checksum(c["hidden"], c["weight"])
    idx, prob = routing.router_topk(g[f"{tag}_logits"], c["k"])
    np.testing.assert_array_equal(idx, g[f"{tag}_idx"])
    np.testing.assert_allclose(prob, g[f"{tag}_prob"], rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("tag", list(inputs.ROUTER_CASES))
def test_dispatch_plan_matches_stable_sort(tag):
    g = golden("router")
    e = inputs.ROUTER_CASES[tag][2]
    plan = routing.dispatch_plan(g[f"{tag}_idx"], e)
    np.testing.assert_array_equal(plan["sort_order"], g[f"{tag}_stable_order"])
    np.testing.assert_array_equal(plan["counts"], g[f"{tag}_counts"])
    # any order the reference's unstable sort returns groups the same routes
    flat = g[f"{tag}_idx"].reshape(-1)
    np.testing.assert_array_equal(flat[g[f"{tag}_unstable_order"]], flat[plan["sort_order"]])


@pytest.mark.parametrize("tag", list(inputs.MOE_CASES))
def test_moe_forward_matches_reference(tag):
    g = golden("moe")
    c = inputs.moe_case(tag)
    assert g[f"{tag}_checksum"] == inputs.checksum(*(c[k] for k in ("flat", "logits", "w_gate", "w_up", "w_down")))
    idx, prob = routing.router_topk(c["logits"], c["k"])
    np.testing.assert_array_equal(idx, g[f"{tag}_idx"])
    out = routing.moe_forward(c["flat"], idx, prob, c["w_gate"], c["w_up"], c["w_down"])
    np.testing.assert_allclose(out, g[f"{tag}_out"], rtol=1e-4, atol=1e-5)


def test_topk_tie_break_is_lowest_index():
    logits = np.array([[0.5, 1.0, 1.0, 0.2, 1.0]], dtype=np.float32)
    idx, _ = routing.router_topk(logits, 3)
    assert idx.tolist() == [[1, 2, 4]]


def test_zipf_bias_is_a_log_distribution():
    b = routing.zipf_expert_bias(32)
    assert b.shape == (32,)
    np.testing.assert_allclose(np.exp(b.astype(np.float64)).sum(), 1.0, rtol=1e-6)
