"""GPU: the state writes a prompt leaves behind -- CSA decode rings, GDN conv
histories, the whole-state zeroing -- against the PyTorch indexing they
replace (bit-exact: they only move bytes)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ring_ref(k, v, kc, vc):
    """The indexed assignment the ring write replaces (model/model.py prefill)."""
    t, w = k.shape[1], kc.shape[1]
    lo = max(0, t - w)
    slots = torch.arange(lo, t, device=k.device) % w
    kc[:, slots] = k[:, lo:t]
    vc[:, slots] = v[:, lo:t]


@pytest.mark.parametrize("b,t,w,kw,vw", [(2, 5, 8, 64, 96), (1, 8, 8, 768, 768),
                                         (3, 21, 8, 64, 40), (2, 300, 128, 24, 20),
                                         (1, 1, 4, 8, 8)])
def test_csa_ring_write_matches_indexing(cuda, b, t, w, kw, vw):
    from hybrid_llm_b200 import kernels
    g = torch.Generator(device="cuda").manual_seed(b * 1000 + t)
    # k and v as column slices of one fused projection, as the prefill has them
    proj = torch.randn(b, t, 16 + kw + vw, device="cuda", generator=g).bfloat16()
    k, v = proj[..., 16:16 + kw], proj[..., 16 + kw:]
    kc0 = torch.randn(b, w, kw, device="cuda", generator=g).bfloat16()
    vc0 = torch.randn(b, w, vw, device="cuda", generator=g).bfloat16()
    kc, vc = kc0.clone(), vc0.clone()
    kernels.csa_ring_write(k, v, kc, vc)
    _ring_ref(k, v, kc0, vc0)
    torch.cuda.synchronize()
    assert torch.equal(kc, kc0) and torch.equal(vc, vc0)


@pytest.mark.parametrize("b,t,d", [(2, 1, 64), (1, 2, 768), (3, 3, 24), (2, 37, 768), (1, 9, 20)])
def test_gdn_history_set_matches_slice_assignment(cuda, b, t, d):
    from hybrid_llm_b200 import kernels
    g = torch.Generator(device="cuda").manual_seed(t * 10 + d)
    x = torch.randn(b, t, d, device="cuda", generator=g).bfloat16()
    hist = torch.randn(b, 3, d, device="cuda", generator=g).bfloat16()
    ref = torch.zeros_like(hist)
    keep = min(t, 3)
    ref[:, 3 - keep:] = x[:, t - keep:]
    kernels.gdn_history_set(x, hist)
    torch.cuda.synchronize()
    assert torch.equal(hist, ref)


def test_zero_regions_clears_exactly_the_regions(cuda):
    from hybrid_llm_b200 import kernels
    buf = torch.full((4096,), 7, dtype=torch.uint8, device="cuda")
    # unaligned starts and odd sizes, a large aligned region and an empty one
    regions = [buf[3:40], buf[100:1124], buf[2000:2001], buf[2048:4000], buf[4001:4001]]
    table, mx = kernels.region_table(regions, buf.device)
    kernels.zero_regions(table, mx)
    torch.cuda.synchronize()
    ref = torch.full((4096,), 7, dtype=torch.uint8)
    for a, e in ((3, 40), (100, 1124), (2000, 2001), (2048, 4000)):
        ref[a:e] = 0
    assert torch.equal(buf.cpu(), ref)


def test_state_zero_clears_every_tensor(cuda):
    from hybrid_llm_b200.config import small_llmy_config
    from hybrid_llm_b200.state import RecurrentState
    st = RecurrentState(small_llmy_config(), 2, "cuda")
    st.fill_synthetic(position=17, seed=1)
    st.zero_()
    st.zero_()  # the cached region table is reused
    torch.cuda.synchronize()
    tensors = [t for _, table in st._tables() for t in table.values()] + [st.positions]
    assert all(int(torch.count_nonzero(t)) == 0 for t in tensors)
