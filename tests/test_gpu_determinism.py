"""GPU: the warp-specialised tensor-core kernels are deterministic.

Each kernel below hands data between warps (and, for the CSA probability
tiles, between the CTAs of a cluster) through shared memory, TMEM and
mbarriers.  A missing wait or an aliased exchange buffer shows up as results
that change from one call to the next, usually long before it shows up as a
tolerance failure, so every case runs the same call several times and
requires identical bits.  The shapes select each kernel variant: the GDN
64-column scan and the value-lane scan, the CSA prefill with and without the
head-splitting cluster, the per-head banded attention with head dims 64 and
128 and more units than SMs, and the grouped GEMMs at 256-row (CTA pair) and 128-row tiles.
"""
import numpy as np
import pytest
import torch

from oracle import gdn

pytestmark = pytest.mark.gpu

REPEATS = 5


def _bf(a):
    return torch.from_numpy(np.asarray(a, dtype=np.float32)).to(torch.bfloat16).cuda()


@pytest.mark.parametrize("b,t,h,kd,vd", [(2, 513, 4, 128, 128), (1, 300, 3, 64, 64),
                                         (5, 260, 16, 128, 128), (5, 200, 16, 64, 128)])
def test_gdn_prefill_repeats_bit_for_bit(cuda, b, t, h, kd, vd):
    """Output and final state of the chunked scan (64-column and value-lane)."""
    from hybrid_llm_b200 import kernels
    rng = np.random.default_rng(t + h)
    q = _bf(gdn.l2norm_heads(rng.normal(size=(b, t, h, kd))))
    k = _bf(gdn.l2norm_heads(rng.normal(size=(b, t, h, kd))))
    v = _bf(rng.normal(size=(b, t, h, vd)))
    beta = _bf(rng.uniform(0, 1, (b, t, h)))
    gate = _bf(rng.uniform(0, 1, (b, t, h, vd)))
    la = torch.from_numpy(rng.uniform(-0.1, 0, (b, t, h)).astype(np.float32)).cuda()
    reset = torch.from_numpy(rng.uniform(size=(b, t)) < 0.02).cuda()
    s0 = torch.from_numpy(rng.normal(0, 0.3, (b, h, kd, vd)).astype(np.float32)).cuda()
    first = None
    for _ in range(REPEATS):
        st = s0.clone()
        out = kernels.gdn_prefill(q, k, v, gate, beta, st, log_alpha=la, reset=reset)
        kernels.check_device_status()
        if first is None:
            first = (out.clone(), st.clone())
        else:
            assert torch.equal(out, first[0]) and torch.equal(st, first[1])


@pytest.mark.parametrize("b,t,h,dh,dm,w", [(1, 512, 12, 64, 768, 512), (3, 1000, 4, 128, 512, 333),
                                           (8, 1024, 8, 64, 512, 256)])
def test_csa_local_prefill_repeats_bit_for_bit(cuda, b, t, h, dh, dm, w):
    """Few units (the probability tiles split each unit's heads over a CTA
    cluster and sum partials over distributed shared memory) and many units."""
    from hybrid_llm_b200 import kernels
    rng = np.random.default_rng(t + h + b)
    q, k = _bf(rng.normal(size=(b, t, h, dh))), _bf(rng.normal(size=(b, t, h, dh)))
    v = _bf(rng.normal(size=(b, t, dm)))
    first = kernels.csa_local_prefill(q, k, v, w)
    kernels.check_device_status()
    for _ in range(REPEATS - 1):
        again = kernels.csa_local_prefill(q, k, v, w)
        kernels.check_device_status()
        assert torch.equal(again, first)


@pytest.mark.parametrize("b,t,h,d,w", [(2, 2048, 8, 64, 512), (8, 1024, 16, 128, 1024)])
def test_banded_attention_repeats_bit_for_bit(cuda, b, t, h, d, w):
    from hybrid_llm_b200 import kernels
    g = torch.Generator(device="cuda").manual_seed(b * t + w)
    q, k, v = (torch.randn(b, t, h, d, device="cuda", generator=g).bfloat16() for _ in range(3))
    q[:, ::61] *= 8  # running-max rescales mid-band
    first = kernels.banded_attention(q, k, v, w)
    kernels.check_device_status()
    assert bool(torch.isfinite(first.float()).all())
    for _ in range(REPEATS - 1):
        again = kernels.banded_attention(q, k, v, w)
        kernels.check_device_status()
        assert torch.equal(again, first)


@pytest.mark.parametrize("tile_m", [256, 128])
def test_grouped_experts_repeat_bit_for_bit(cuda, tile_m):
    """The SwiGLU / probability GEMMs over a skewed plan (16,384 routes, 32
    experts, top-4): CTA-pair 256 x 256 tiles and single-CTA 128 x 256 tiles."""
    from hybrid_llm_b200 import kernels
    n, d, e, k, f = 4096, 1024, 32, 4, 512
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(n, d, device="cuda", generator=g).bfloat16()
    logits = torch.randn(n, e, device="cuda", generator=g)
    logits[:, :4] += 2.0  # a few heavy experts
    w13 = kernels.pack_w13(*((torch.randn(e, f, d, device="cuda", generator=g) * 0.02).bfloat16()
                             for _ in range(2)))
    wd = (torch.randn(e, d, f, device="cuda", generator=g) * 0.02).bfloat16()
    plan = kernels.route(logits, k, tile_m=tile_m)
    rows = n * k
    scratch = torch.empty(kernels.grouped_scratch_bytes(rows, d, f), dtype=torch.uint8,
                          device="cuda")
    outs = []
    for _ in range(REPEATS):
        y = torch.empty(rows, d, device="cuda", dtype=torch.bfloat16)
        kernels.moe_grouped_experts_to(x, rows, plan.perm_token, plan.perm_prob, plan.offsets,
                                       plan.tile_offsets, plan.tile_m, w13, wd, scratch, y)
        kernels.check_device_status()
        outs.append(y)
    assert int(plan.tile_m) == tile_m
    for y in outs[1:]:
        assert torch.equal(y, outs[0])
