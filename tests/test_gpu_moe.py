"""GPU: tcgen05 grouped SwiGLU experts vs the fp64 oracle and a torch fp32 reference."""
import numpy as np
import pytest
import torch

from oracle import routing

pytestmark = pytest.mark.gpu

# bf16 tolerance for the routed output: the kernel rounds the SwiGLU
# activation and every routed row to bf16 and sums the k rows in fp32.
MAX_REL = 2e-2   # max |out - ref| / max |ref|
MEAN_REL = 5e-3  # mean |out - ref| / mean |ref|


def _case(n, d, e, k, f, seed, zipf=False):
    rng = np.random.default_rng(seed)
    bf = lambda a: torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16)
    x = bf(rng.normal(0, 1, (n, d)))
    logits = rng.normal(0, 0.64, (n, e)).astype(np.float32)
    bias = routing.zipf_expert_bias(e) if zipf else None
    wg = bf(rng.normal(0, 0.02, (e, f, d)))
    wu = bf(rng.normal(0, 0.02, (e, f, d)))
    wd = bf(rng.normal(0, 0.02, (e, d, f)))
    return x, logits, bias, wg, wu, wd


def _run(x, logits, bias, wg, wu, wd, k, path="auto"):
    from hybrid_llm_b200 import kernels
    dev = "cuda"
    tile_m = 128 if path == "grouped128" else kernels.TILE_M
    if path == "grouped128":
        path = "grouped"
    plan = kernels.route(torch.from_numpy(logits).to(dev), k,
                         None if bias is None else torch.from_numpy(bias).to(dev), tile_m=tile_m)
    w13 = kernels.pack_w13(wg.to(dev), wu.to(dev))
    out = kernels.moe_grouped(x.to(dev), plan, w13, wd.to(dev), path=path)
    torch.cuda.synchronize()
    kernels.check_device_status()
    return out, plan


def _errors(out, ref):
    out = out.float().cpu().numpy().astype(np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(out - ref)
    return err.max() / np.abs(ref).max(), err.mean() / np.abs(ref).mean()


@pytest.mark.parametrize("path", ["grouped", "grouped128", "decode"])
@pytest.mark.parametrize("n,d,e,k,f", [(300, 256, 8, 2, 128), (1, 768, 16, 2, 1024),
                                       (5, 512, 8, 2, 1024), (700, 256, 4, 4, 256),
                                       (129, 1024, 32, 4, 512), (64, 2048, 64, 8, 1024)])
def test_moe_matches_oracle(cuda, n, d, e, k, f, path):
    x, logits, bias, wg, wu, wd = _case(n, d, e, k, f, seed=n + d)
    out, plan = _run(x, logits, bias, wg, wu, wd, k, path=path)
    idx, prob = routing.router_topk(logits, k, bias)
    ref = routing.moe_forward(x.float().numpy(), idx, prob, wg.float().numpy(),
                              wu.float().numpy(), wd.float().numpy())
    mx, mean = _errors(out, ref)
    assert mx < MAX_REL and mean < MEAN_REL, (mx, mean)


def _torch_reference(x, plan, wg, wu, wd):
    """fp32 torch restatement of moe.py:72-81 on the GPU (per-expert matmuls)."""
    xf = x.float()
    out = torch.zeros_like(xf)
    idx, prob = plan.topk_idx, plan.topk_prob
    for e in range(wg.shape[0]):
        tok, slot = torch.nonzero(idx == e, as_tuple=True)
        if tok.numel() == 0:
            continue
        h = torch.nn.functional.silu(xf[tok] @ wg[e].float().T) * (xf[tok] @ wu[e].float().T)
        out.index_add_(0, tok, (h @ wd[e].float().T) * prob[tok, slot, None])
    return out


@pytest.mark.parametrize("path", ["grouped", "grouped128"])
def test_moe_isolated_layer_full_size(cuda, path):
    """16384 tokens x 1024, 32 experts top-4, F=512, Zipf-skewed routing."""
    x, logits, bias, wg, wu, wd = _case(16384, 1024, 32, 4, 512, seed=3, zipf=True)
    dev = "cuda"
    out, plan = _run(x, logits, bias, wg, wu, wd, 4, path=path)
    ref = _torch_reference(x.to(dev), plan, wg.to(dev), wu.to(dev), wd.to(dev))
    err = (out.float() - ref).abs()
    assert float(err.max() / ref.abs().max()) < MAX_REL
    assert float(err.mean() / ref.abs().mean()) < MEAN_REL
    counts = plan.counts.cpu()
    assert int(counts.sum()) == 16384 * 4 and int(counts.max()) > 4 * int(counts.min() + 1)


def test_moe_repeated_calls_identical(cuda):
    x, logits, bias, wg, wu, wd = _case(513, 512, 8, 2, 256, seed=9)
    a, _ = _run(x, logits, bias, wg, wu, wd, 2)
    b, _ = _run(x, logits, bias, wg, wu, wd, 2)
    assert torch.equal(a, b)


@pytest.mark.parametrize("grouped", [True, False])
@pytest.mark.parametrize("n,d,e,k,f", [(64, 2048, 64, 8, 1024), (37, 512, 8, 2, 384),
                                       (300, 256, 16, 4, 256)])
def test_moe_expert_rows_match_oracle(cuda, n, d, e, k, f, grouped):
    """Per-route expert rows (decode-batch path) combined by the routed residual add."""
    from hybrid_llm_b200 import kernels
    x, logits, bias, wg, wu, wd = _case(n, d, e, k, f, seed=11 + n)
    plan = kernels.route(torch.from_numpy(logits).to(cuda), k, tile_m=128)
    w13 = kernels.pack_w13(wg.to(cuda), wu.to(cuda))
    xd, wdd = x.to(cuda), wd.to(cuda)
    rows = plan.perm_token.numel()
    if grouped:
        y = torch.empty(rows, d, dtype=torch.bfloat16, device=cuda)
        scratch = torch.empty(kernels.grouped_scratch_bytes(rows, d, f), dtype=torch.uint8,
                              device=cuda)
        kernels.moe_grouped_experts_to(xd, rows, plan.perm_token, plan.perm_prob, plan.offsets,
                                       plan.tile_offsets, 128, w13, wdd, scratch, y)
    else:
        y = kernels.moe_decode_experts(xd, plan, w13, wdd)
    streams = torch.zeros(n, d, dtype=torch.float32, device=cuda)
    kernels.add_rmsnorm_routed(streams, y, plan, None, 1e-6, normalize=False)
    torch.cuda.synchronize()
    kernels.check_device_status()
    idx, prob = routing.router_topk(logits, k, None)
    ref = routing.moe_forward(x.float().numpy(), idx, prob, wg.float().numpy(),
                              wu.float().numpy(), wd.float().numpy())
    mx, mean = _errors(streams, ref)
    assert mx < MAX_REL and mean < MEAN_REL, (mx, mean)
    # the row map: writing row pos to out_row[pos] permutes the rows exactly
    if grouped:
        perm = torch.randperm(rows, device=cuda).to(torch.int32)
        y2 = torch.empty_like(y)
        kernels.moe_grouped_experts_to(xd, rows, plan.perm_token, plan.perm_prob, plan.offsets,
                                       plan.tile_offsets, 128, w13, wdd, scratch, y2, perm)
        assert torch.equal(y2[perm.long()], y)
