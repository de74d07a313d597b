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


def _decode_router_inputs(n, d, e, seed):
    rng = np.random.default_rng(seed)
    streams = rng.normal(0, 1, (n, d)).astype(np.float32)
    delta = rng.normal(0, 0.5, (n, d)).astype(np.float32)
    ffn_w = rng.uniform(0.5, 1.5, d).astype(np.float32)
    rn_w = rng.uniform(0.5, 1.5, d).astype(np.float32)
    w_r = rng.normal(0, 0.02, (e, d)).astype(np.float32)
    return streams, delta, ffn_w, rn_w, w_r


def _decode_route(fn, streams, delta, ffn_w, rn_w, w_r, k, eps=1e-6):
    from hybrid_llm_b200 import kernels
    st = torch.from_numpy(streams).cuda()
    dl = torch.from_numpy(delta).cuda().bfloat16()
    m_bf = torch.empty(st.shape, dtype=torch.bfloat16, device="cuda")
    plan = fn(st, dl, torch.from_numpy(ffn_w).cuda(), torch.from_numpy(rn_w).cuda(),
              torch.from_numpy(w_r).cuda(), k, eps, m_bf, tile_m=128)
    torch.cuda.synchronize()
    return st, m_bf, plan


@pytest.mark.parametrize("n,d,e,k", [(1, 768, 16, 2), (4, 512, 64, 8), (16, 2048, 16, 2)])
def test_route_decode_matches_single_cta(cuda, n, d, e, k):
    """The multi-CTA decode router equals the one-CTA fused router bit for bit."""
    from hybrid_llm_b200 import kernels
    args = _decode_router_inputs(n, d, e, seed=n + e)
    a = _decode_route(lambda *x, **kw: kernels.route_fused(*x, **kw, variant="single"), *args, k)
    b = _decode_route(kernels.route_decode, *args, k)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    for f in ("topk_idx", "topk_prob", "counts", "offsets", "tile_offsets", "perm_token",
              "perm_prob", "route_pos"):
        assert torch.equal(getattr(a[2], f), getattr(b[2], f)), f


@pytest.mark.parametrize("n,d,e,k", [(64, 2048, 64, 8), (256, 768, 16, 2), (33, 1024, 256, 32)])
def test_route_decode_matches_oracle(cuda, n, d, e, k):
    """Residual add, the two RMSNorms and the fp32 router logits against fp64:
    indices equal wherever the k-th and (k+1)-th logits are not within 1e-4."""
    from hybrid_llm_b200 import kernels
    streams, delta, ffn_w, rn_w, w_r = _decode_router_inputs(n, d, e, seed=7 * n + d)
    st, m_bf, plan = _decode_route(kernels.route_fused, streams, delta, ffn_w, rn_w, w_r, k)
    x = streams.astype(np.float64) + torch.from_numpy(delta).bfloat16().double().numpy()
    np.testing.assert_allclose(st.cpu().numpy(), x, rtol=1e-6, atol=1e-6)
    m = x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6) * ffn_w
    np.testing.assert_allclose(m_bf.float().cpu().numpy(), m, rtol=1e-2, atol=1e-2)
    r = m / np.sqrt((m * m).mean(-1, keepdims=True) + 1e-6) * rn_w
    logits = r @ w_r.astype(np.float64).T
    idx, prob = routing.router_topk(logits.astype(np.float32), k)
    got = plan.topk_idx.cpu().numpy()
    srt = -np.sort(-logits, axis=-1)
    clear = (srt[:, k - 1] - srt[:, k]) > 1e-4 if k < e else np.ones(n, bool)
    assert clear.mean() > 0.8
    np.testing.assert_array_equal(np.sort(got[clear], -1), np.sort(idx[clear], -1))
    np.testing.assert_allclose(plan.topk_prob.cpu().numpy()[clear], prob[clear], rtol=1e-4,
                               atol=1e-5)
    ref = routing.dispatch_plan(got, e, tile_m=128)
    for f in ("counts", "offsets", "tile_offsets", "perm_token", "route_pos"):
        np.testing.assert_array_equal(getattr(plan, f).cpu().numpy(), ref[f], err_msg=f)
    np.testing.assert_array_equal(plan.perm_prob.cpu().numpy(),
                                  plan.topk_prob.cpu().numpy().reshape(-1)[ref["sort_order"]])


@pytest.mark.parametrize("n,d,e,k", [(512, 768, 16, 2), (3000, 1024, 64, 8), (7, 256, 8, 2),
                                     (1, 128, 4, 1), (1100, 512, 32, 2)])
def test_route_norm_matches_norm_then_route(cuda, n, d, e, k):
    """llmyb_route_norm (router RMSNorm + fp32 logits + top-k in one kernel, then
    the plan): logits within fp32 rounding of an fp64 RMSNorm + F.linear, and
    the routing and plan bit-identical to llmyb_route on those logits (one CTA
    plan up to 2048 routes, the chunked plan above)."""
    from hybrid_llm_b200 import kernels
    g = torch.Generator(device=cuda).manual_seed(n + d)
    m = torch.randn(n, d, device=cuda, generator=g)
    rn = 1 + 0.1 * torch.randn(d, device=cuda, generator=g)
    w = 0.02 * torch.randn(e, d, device=cuda, generator=g)
    lg = torch.empty(n, e, device=cuda)
    plan = kernels.route_norm(m, rn, w, k, 1e-6, tile_m=128, logits_out=lg)
    md = m.double()
    r = md * torch.rsqrt(md.pow(2).mean(-1, keepdim=True) + 1e-6) * rn.double()
    ref = r @ w.double().t()
    err = float((lg.double() - ref).abs().max() / ref.abs().max())
    assert err < 1e-5, err
    want = kernels.route(lg, k, tile_m=128)
    for name in ("topk_idx", "topk_prob", "counts", "offsets", "tile_offsets", "perm_token",
                 "perm_prob", "route_pos"):
        assert torch.equal(getattr(plan, name), getattr(want, name)), name


@pytest.mark.parametrize("n,e,k", [(512, 16, 2), (1000, 64, 2), (300, 7, 3), (33, 64, 2),
                                   (256, 8, 8), (1024, 32, 2)])
def test_single_cta_plan_equals_chunked_plan(cuda, n, e, k):
    """The one-CTA plan of llmyb_route (up to 2048 routes; the permutation
    spread over all warps for E <= 64) gives the chunked multi-CTA plan of
    llmyb_moe_plan on the same routes, field by field."""
    from hybrid_llm_b200 import kernels
    g = torch.Generator(device=cuda).manual_seed(n * e + k)
    logits = torch.randn(n, e, device=cuda, generator=g)
    logits[: n // 3] = logits[: n // 3].round()  # ties between experts
    small = kernels.route(logits, k, tile_m=128, with_sort_order=True)
    chunked = kernels.moe_plan(small.topk_idx, small.topk_prob, e, tile_m=128,
                               with_sort_order=True)
    for name in ("counts", "offsets", "tile_offsets", "perm_token", "perm_prob", "route_pos",
                 "sort_order"):
        assert torch.equal(getattr(small, name), getattr(chunked, name)), name
