"""The reference-hook replacements: installation (CPU) and results (GPU)."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import attention, gdn, routing, sampling


def test_install_sets_every_reference_hook():
    from hybrid_llm_b200 import seams
    moe = SimpleNamespace(_triton_moe_dispatch=None, _triton_available=False)
    g = SimpleNamespace(_triton_gdn_scan=None, _triton_gdn_step=None, _triton_gdn_available=False,
                        _fused_gdn_scan=object(), _fused_gdn_step=object())
    band = SimpleNamespace(triton_banded_local_attention=None)
    seams.install(moe, g, band)
    assert moe._triton_moe_dispatch is seams.triton_moe_dispatch and moe._triton_available
    assert g._triton_gdn_scan is seams.triton_gdn_scan and g._triton_gdn_step is seams.triton_gdn_step
    assert g._triton_gdn_available and g._fused_gdn_scan is None
    assert band.triton_banded_local_attention is seams.triton_banded_local_attention


def test_seams_refuse_cpu_tensors():
    from hybrid_llm_b200 import seams
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        seams.router_topk(torch.zeros(4, 8), 2)


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.abs(a - b).max() / np.abs(b).max()


@pytest.mark.gpu
def test_moe_dispatch_seam(cuda):
    from hybrid_llm_b200 import seams
    rng = np.random.default_rng(0)
    n, d, e, k, f = 200, 256, 8, 2, 128
    flat = torch.from_numpy(rng.normal(size=(n, d)).astype(np.float32)).cuda()
    logits = rng.normal(size=(n, e)).astype(np.float32)
    vals, idx = torch.topk(torch.from_numpy(logits).cuda(), k)
    prob = vals.softmax(-1)
    wg, wu = (torch.from_numpy(rng.normal(0, 0.05, (e, f, d)).astype(np.float32)).cuda() for _ in range(2))
    wd = torch.from_numpy(rng.normal(0, 0.05, (e, d, f)).astype(np.float32)).cuda()
    out = seams.triton_moe_dispatch(flat, idx, prob, e, wg, wu, wd)
    assert out.dtype == flat.dtype and out.shape == flat.shape
    ref = routing.moe_forward(flat.cpu().numpy(), idx.cpu().numpy(), prob.cpu().numpy(),
                              wg.cpu().numpy(), wu.cpu().numpy(), wd.cpu().numpy())
    assert _rel(out.cpu().numpy(), ref) < 2e-2


@pytest.mark.gpu
def test_gdn_scan_and_step_seams(cuda):
    from hybrid_llm_b200 import seams
    rng = np.random.default_rng(1)
    b, t, h, kd, vd = 2, 70, 2, 64, 64
    q = torch.from_numpy(gdn.l2norm_heads(rng.normal(size=(b, t, h, kd))).astype(np.float32)).cuda()
    k = torch.from_numpy(gdn.l2norm_heads(rng.normal(size=(b, t, h, kd))).astype(np.float32)).cuda()
    v = torch.from_numpy(rng.normal(size=(b, t, h, vd)).astype(np.float32)).cuda()
    beta = torch.rand(b, t, h, 1, device="cuda")
    gate = torch.rand(b, t, h, vd, device="cuda")
    reset = torch.zeros(b, t, dtype=torch.bool, device="cuda")
    dl = torch.full((h,), 2.0, device="cuda")
    st = torch.zeros(b, h, kd, vd, device="cuda")
    out, final = seams.triton_gdn_scan(q, k, v, beta, gate, reset, dl, st)
    assert torch.count_nonzero(st) == 0  # the caller's state is not modified
    f = lambda x: x.float().cpu().numpy()
    o_ref, s_ref = gdn.gdn_recurrent(f(q), f(k), f(v), f(beta), f(gate), None,
                                     gdn.sigmoid(f(dl)), np.zeros((b, h, kd, vd)))
    assert _rel(f(out), o_ref) < 2e-2 and _rel(f(final), s_ref) < 1e-2
    o1, s1 = seams.triton_gdn_step(q[:, :1], k[:, :1], v[:, :1], beta[:, :1], gate[:, :1],
                                   reset[:, :1], dl, final)
    assert s1 is final and o1.shape == (b, 1, h, vd)


@pytest.mark.gpu
def test_banded_attention_seam_shared_value_stream(cuda):
    from hybrid_llm_b200 import seams
    rng = np.random.default_rng(2)
    b, t, h, d, dm, w = 1, 90, 4, 64, 256, 32
    q, k = (torch.from_numpy(rng.normal(size=(b, t, h, d)).astype(np.float32)).cuda() for _ in range(2))
    v = torch.from_numpy(rng.normal(size=(b, t, dm)).astype(np.float32)).cuda()
    per_head = seams.triton_banded_local_attention(q, k, v.unsqueeze(2), window_size=w)
    assert per_head.shape == (b, t, h, dm)
    ref = attention.csa_local(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), w)
    assert _rel(per_head.mean(2).cpu().numpy(), ref) < 2e-2
    assert _rel(seams.csa_local_attention(q, k, v, w).cpu().numpy(), ref) < 2e-2


@pytest.mark.gpu
def test_router_and_sampler_seams(cuda):
    from hybrid_llm_b200 import seams
    rng = np.random.default_rng(3)
    logits = rng.normal(size=(3, 5, 16)).astype(np.float32)
    idx, prob = seams.router_topk(torch.from_numpy(logits).cuda(), 2)
    ref_idx, _ = routing.router_topk(logits.reshape(-1, 16), 2)
    assert np.array_equal(idx.cpu().numpy().reshape(-1, 2), ref_idx) and idx.shape == (3, 5, 2)
    lg = rng.normal(size=(2, 100)).astype(np.float32)
    tok, lp = seams.sample_next_token(torch.from_numpy(lg).cuda(), [3, 5], temp=0.0, top_k=0,
                                      top_p=1.0, rep=1.1)
    ref, _ = sampling.sample_next_token(lg, [[3, 5], [3, 5]], temp=0.0, top_k=0, top_p=1.0,
                                        rep=1.1, uniforms=[0.5, 0.5])
    assert tok.view(-1).cpu().tolist() == ref.tolist()
