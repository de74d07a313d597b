"""GPU: banded attention (per-head and CSA head-averaged) and CSA decode vs the oracle."""
import numpy as np
import pytest
import torch

import inputs
from conftest import golden
from oracle import attention

pytestmark = pytest.mark.gpu

REL = 2e-2  # bf16 inputs/outputs, fp32 accumulation; relative to max |ref|


def _bf(a):
    return torch.from_numpy(np.asarray(a, dtype=np.float32)).to(torch.bfloat16)


def _f(t):
    return t.float().cpu().numpy().astype(np.float64)


def _rel(got, ref):
    return np.abs(got - ref).max() / np.abs(ref).max()


@pytest.mark.parametrize("b,t,h,d,w,hv", [(2, 200, 3, 64, 50, 3), (1, 130, 2, 128, 128, 1),
                                          (1, 64, 4, 64, 1000, 4), (3, 1, 2, 128, 16, 2),
                                          (1, 517, 2, 128, 64, 2), (2, 300, 1, 64, 300, 1)])
def test_banded_attention_matches_oracle(cuda, b, t, h, d, w, hv):
    from hybrid_llm_b200 import kernels
    rng = np.random.default_rng(t + d)
    q, k = _bf(rng.normal(size=(b, t, h, d))), _bf(rng.normal(size=(b, t, h, d)))
    v = _bf(rng.normal(size=(b, t, hv, d)))
    out = kernels.banded_attention(q.cuda(), k.cuda(), v.cuda(), w)
    kernels.check_device_status()
    ref = attention.banded_attention(_f(q), _f(k), _f(v), w)
    assert _rel(_f(out), ref) < REL


def _torch_band(q, k, v, w):
    """fp32 dense-masked softmax attention on the GPU: q,k [B,T,H,D], v [B,T,H|1,D]."""
    qf, kf, vf = (x.float().transpose(1, 2) for x in (q, k, v))
    t = q.shape[1]
    i = torch.arange(t, device=q.device)
    vis = (i[None, :] <= i[:, None]) & (i[:, None] - i[None, :] < w)
    s = (qf @ kf.transpose(-1, -2)) * q.shape[-1] ** -0.5
    s = s.masked_fill(~vis, float("-inf"))
    return (torch.softmax(s, -1) @ vf).transpose(1, 2)


@pytest.mark.parametrize("b,t,h,d,w,hv", [(4, 2048, 8, 64, 700, 1), (3, 1500, 8, 128, 256, 8),
                                          (2, 1024, 20, 128, 128, 20), (1, 4096, 2, 128, 4096, 2)])
def test_banded_attention_many_units_per_cta(cuda, b, t, h, d, w, hv):
    """More (row, head, query-tile) units than SMs: the persistent loop, the
    double-buffered Q tiles and the running-max rescale across units."""
    from hybrid_llm_b200 import kernels
    g = torch.Generator(device="cuda").manual_seed(t + w)
    q, k = (torch.randn(b, t, h, d, device="cuda", generator=g).bfloat16() for _ in range(2))
    v = torch.randn(b, t, hv, d, device="cuda", generator=g).bfloat16()
    # a few large scores so that the running max moves by more than 2^8 mid-band
    q[:, ::97] *= 6
    out = kernels.banded_attention(q, k, v, w)
    kernels.check_device_status()
    ref = _torch_band(q, k, v, w)
    err = (out.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < REL, err
    # the kernel is deterministic: repeated calls give the same bits (a race
    # between the softmax warps' shared-memory exchanges would show up here)
    for _ in range(4):
        again = kernels.banded_attention(q, k, v, w)
        kernels.check_device_status()
        assert torch.equal(again, out)


@pytest.mark.parametrize("tag", list(inputs.BAND_CASES))
def test_banded_attention_on_reference_golden_inputs(cuda, tag):
    """Padded to a supported head dim with zeros (q.k and the output unchanged)."""
    from hybrid_llm_b200 import kernels
    g = golden("band")
    c = inputs.band_case(tag)
    pad = lambda a: np.concatenate([a, np.zeros(a.shape[:-1] + (64 - a.shape[-1],), np.float32)], -1)
    d = c["q"].shape[-1]
    out = kernels.banded_attention(_bf(pad(c["q"])).cuda(), _bf(pad(c["k"])).cuda(),
                                   _bf(pad(c["v"])).cuda(), c["window"], scale=d ** -0.5)
    torch.cuda.synchronize()
    assert _rel(_f(out)[..., :c["v"].shape[-1]], g[f"{tag}_out"]) < REL


def test_banded_attention_long_context_full_size(cuda):
    """B=8, T=8192, H=16, D=128, W=1024: oracle on sampled rows of two heads."""
    from hybrid_llm_b200 import kernels
    b, t, h, d, w = 8, 8192, 16, 128, 1024
    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v = (torch.randn(b, t, h, d, device="cuda", generator=g).bfloat16() for _ in range(3))
    out = kernels.banded_attention(q, k, v, w)
    kernels.check_device_status()
    rows = np.array([0, 1, 63, 64, 1023, 1024, 1025, 4000, 8191])
    for bi, hi in [(0, 0), (7, 15)]:
        qq = _f(q[bi, rows, hi])
        kk, vv = _f(k[bi, :, hi]), _f(v[bi, :, hi])
        ref = np.empty((rows.size, d))
        for n, r in enumerate(rows):
            lo = max(0, r - w + 1)
            s = kk[lo:r + 1] @ qq[n] / np.sqrt(d)
            p = np.exp(s - s.max())
            ref[n] = (p / p.sum()) @ vv[lo:r + 1]
        assert _rel(_f(out[bi, rows, hi]), ref) < REL


@pytest.mark.parametrize("b,t,h,dh,dm,w", [(1, 256, 8, 64, 512, 128), (1, 512, 12, 64, 768, 512),
                                           (2, 100, 4, 128, 256, 40), (1, 70, 16, 128, 2048, 2048),
                                           (1, 5, 2, 64, 128, 128), (1, 300, 3, 64, 384, 100),
                                           (3, 1000, 4, 128, 512, 333), (2, 700, 6, 64, 768, 129),
                                           (1, 384, 2, 64, 192, 1000)])
def test_csa_local_prefill_matches_oracle(cuda, b, t, h, dh, dm, w):
    """Head dim 64 / 128 with D % 128 == 0 on the tcgen05 kernels (ragged last
    query tiles, windows shorter and longer than the sequence, W - 1 a multiple
    of 128); D = 192 on the mma.sync kernels."""
    from hybrid_llm_b200 import kernels
    rng = np.random.default_rng(t + h)
    q, k = _bf(rng.normal(size=(b, t, h, dh))), _bf(rng.normal(size=(b, t, h, dh)))
    v = _bf(rng.normal(size=(b, t, dm)))
    out = kernels.csa_local_prefill(q.cuda(), k.cuda(), v.cuda(), w)
    torch.cuda.synchronize()
    ref = attention.csa_local(_f(q), _f(k), _f(v), w)
    assert _rel(_f(out), ref) < REL


@pytest.mark.parametrize("b,h,dh,dm,w,pos", [(1, 12, 64, 768, 512, 700), (3, 8, 64, 512, 128, 5),
                                              (64, 16, 128, 2048, 2048, 4100),
                                              (2, 4, 128, 256, 40, 39), (1, 2, 64, 128, 16, 0)])
def test_csa_local_decode_matches_oracle(cuda, b, h, dh, dm, w, pos):
    from hybrid_llm_b200 import kernels
    rng = np.random.default_rng(b * w + pos)
    hd = h * dh
    # history of tokens 0..pos-1 in the ring, current token `pos`
    kc = _bf(rng.normal(size=(b, w, hd)))
    vc = _bf(rng.normal(size=(b, w, dm)))
    q = _bf(rng.normal(size=(b, hd)))
    kn, vn = _bf(rng.normal(size=(b, hd))), _bf(rng.normal(size=(b, dm)))
    positions = torch.full((b,), pos, dtype=torch.int32)
    kcd, vcd = kc.clone().cuda(), vc.clone().cuda()
    out = kernels.csa_local_decode(q.cuda(), kn.cuda(), vn.cuda(), kcd, vcd, positions.cuda(), h)
    torch.cuda.synchronize()
    slot = pos % w
    kf, vf = _f(kc), _f(vc)
    kf[:, slot], vf[:, slot] = _f(kn), _f(vn)
    n = min(pos + 1, w)
    valid = np.arange(w)[None, :] < n
    ref = attention.csa_local_step(_f(q).reshape(b, h, dh), kf.reshape(b, w, h, dh), vf,
                                   np.broadcast_to(valid, (b, w)))
    assert _rel(_f(out), ref) < REL
    assert torch.equal(kcd[:, slot].cpu(), kn) and torch.equal(vcd[:, slot].cpu(), vn)


@pytest.mark.parametrize("h,dh,dm,w", [(12, 64, 768, 512), (4, 128, 256, 40), (16, 128, 2048, 256)])
def test_csa_local_decode_staged_equals_plain(cuda, h, dh, dm, w):
    """Batches of up to 32 rows stage each CTA's ring rows in shared memory
    (512 threads); larger batches read them from global memory (256 threads).
    Same ring updates; outputs equal up to the order of the fp32 value sums
    (at most one bf16 unit in the last place)."""
    from hybrid_llm_b200 import kernels
    b = 40
    rng = np.random.default_rng(h * w)
    hd = h * dh
    kc = _bf(rng.normal(size=(b, w, hd))).cuda()
    vc = _bf(rng.normal(size=(b, w, dm))).cuda()
    q = _bf(rng.normal(size=(b, hd))).cuda()
    kn, vn = _bf(rng.normal(size=(b, hd))).cuda(), _bf(rng.normal(size=(b, dm))).cuda()
    positions = torch.from_numpy(rng.integers(0, 3 * w, b).astype(np.int32)).cuda()
    k1, v1 = kc.clone(), vc.clone()
    plain = kernels.csa_local_decode(q, kn, vn, k1, v1, positions, h)       # 40 rows: plain
    k2, v2 = kc.clone(), vc.clone()
    staged = torch.cat([kernels.csa_local_decode(q[i:i + 8], kn[i:i + 8], vn[i:i + 8],
                                                 k2[i:i + 8], v2[i:i + 8], positions[i:i + 8], h)
                        for i in range(0, b, 8)])                             # 8 rows: staged
    torch.cuda.synchronize()
    kernels.check_device_status()
    ulp = plain.float().abs() * 2.0 ** -7 + 1e-30
    assert bool(((plain.float() - staged.float()).abs() <= ulp).all())
    assert float((plain == staged).float().mean()) > 0.9
    assert torch.equal(k1, k2) and torch.equal(v1, v2)
