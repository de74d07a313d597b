"""GPU: GDN decode step, chunked prefill scan and conv gate vs the fp64 oracle."""
import numpy as np
import pytest
import torch

import inputs
from conftest import golden
from oracle import gdn

pytestmark = pytest.mark.gpu

# bf16 inputs, fp32 state; outputs are rounded to bf16 (as the reference does
# under bf16 autocast).  Tolerances relative to the max magnitude.
OUT_REL = 2e-2
STATE_REL = 5e-3


def _bf(a):
    return torch.from_numpy(np.asarray(a, dtype=np.float32)).to(torch.bfloat16)


def _f(t):
    return t.float().cpu().numpy().astype(np.float64)


def _inputs(b, t, h, kd, vd, seed, per_token=False, resets=True):
    rng = np.random.default_rng(seed)
    q = _bf(gdn.l2norm_heads(rng.normal(size=(b, t, h, kd))))
    k = _bf(gdn.l2norm_heads(rng.normal(size=(b, t, h, kd))))
    v = _bf(rng.normal(size=(b, t, h, vd)))
    beta = _bf(rng.uniform(0, 1, (b, t, h)))
    gate = _bf(rng.uniform(0, 1, (b, t, h, vd)))
    decay_logit = rng.uniform(0.5, 3.0, h).astype(np.float32)
    log_alpha = rng.uniform(-0.1, 0, (b, t, h)).astype(np.float32) if per_token else None
    reset = (rng.uniform(size=(b, t)) < 0.02) if resets else np.zeros((b, t), bool)
    state = rng.normal(0, 0.3, (b, h, kd, vd)).astype(np.float32)
    return q, k, v, beta, gate, decay_logit, log_alpha, reset, state


def _rel(got, ref):
    return np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)


@pytest.mark.parametrize("b,h,kd,vd", [(1, 12, 64, 64), (5, 3, 128, 128), (2, 4, 64, 128),
                                       (64, 16, 128, 128)])
def test_gdn_step_matches_oracle(cuda, b, h, kd, vd):
    from hybrid_llm_b200 import kernels
    q, k, v, beta, gate, dl, _, _, state = _inputs(b, 1, h, kd, vd, seed=b * h + kd)
    reset = np.zeros(b, bool)
    reset[0] = b > 1
    st = torch.from_numpy(state).cuda()
    out = kernels.gdn_step(q[:, 0].cuda(), k[:, 0].cuda(), v[:, 0].cuda(), gate[:, 0].cuda(),
                           beta[:, 0].cuda(), st, decay_logit=torch.from_numpy(dl).cuda(),
                           reset=torch.from_numpy(reset).cuda())
    torch.cuda.synchronize()
    o_ref, s_ref = gdn.gdn_recurrent(_f(q), _f(k), _f(v), _f(beta), _f(gate), reset[:, None],
                                     gdn.sigmoid(dl), state)
    assert _rel(_f(out), o_ref[:, 0]) < OUT_REL
    assert _rel(st.cpu().numpy(), s_ref) < 1e-5


@pytest.mark.parametrize("b,t,h,kd,vd,per_token", [
    (2, 150, 3, 64, 64, False), (1, 300, 2, 128, 128, True), (3, 64, 2, 64, 128, False),
    (1, 1, 2, 128, 64, False), (2, 513, 4, 128, 128, False), (1, 200, 1, 64, 64, True),
    # 2*B*H > SMs: the value-lane scan (one CTA per row and head), K = 64 and 128
    (5, 200, 16, 64, 128, False), (5, 130, 16, 128, 128, True)])
def test_gdn_prefill_matches_oracle(cuda, b, t, h, kd, vd, per_token):
    from hybrid_llm_b200 import kernels
    q, k, v, beta, gate, dl, la, reset, state = _inputs(b, t, h, kd, vd, seed=t + kd, per_token=per_token)
    st = torch.from_numpy(state).cuda()
    out = kernels.gdn_prefill(q.cuda(), k.cuda(), v.cuda(), gate.cuda(), beta.cuda(), st,
                              decay_logit=torch.from_numpy(dl).cuda(),
                              log_alpha=None if la is None else torch.from_numpy(la).cuda(),
                              reset=torch.from_numpy(reset).cuda())
    torch.cuda.synchronize()
    alpha = np.exp(la) if la is not None else gdn.sigmoid(dl)
    o_ref, s_ref = gdn.gdn_recurrent(_f(q), _f(k), _f(v), _f(beta), _f(gate), reset, alpha, state)
    assert _rel(_f(out), o_ref) < OUT_REL
    assert _rel(st.cpu().numpy(), s_ref) < STATE_REL


def test_gdn_prefill_long_context_full_size(cuda):
    """B=8, T=8192, H=16, K=V=128, log-decay U[-0.1,0], beta U[0,1]; oracle on two heads."""
    from hybrid_llm_b200 import kernels
    b, t, h, d = 8, 8192, 16, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.nn.functional.normalize(torch.randn(b, t, h, d, device="cuda", generator=g), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(b, t, h, d, device="cuda", generator=g), dim=-1).bfloat16()
    v = torch.randn(b, t, h, d, device="cuda", generator=g).bfloat16()
    beta = torch.rand(b, t, h, device="cuda", generator=g).bfloat16()
    gate = torch.rand(b, t, h, d, device="cuda", generator=g).bfloat16()
    la = -0.1 * torch.rand(b, t, h, device="cuda", generator=g)
    st = torch.zeros(b, h, d, d, device="cuda")
    out = kernels.gdn_prefill(q, k, v, gate, beta, st, log_alpha=la)
    torch.cuda.synchronize()
    for bi, hi in [(0, 0), (7, 15)]:
        sl = lambda x: _f(x[bi:bi + 1, :, hi:hi + 1])
        o_ref, s_ref = gdn.gdn_recurrent(sl(q), sl(k), sl(v), sl(beta), sl(gate), None,
                                         np.exp(sl(la)), np.zeros((1, 1, d, d)))
        assert _rel(_f(out[bi:bi + 1, :, hi:hi + 1]), o_ref) < OUT_REL
        assert _rel(st[bi:bi + 1, hi:hi + 1].cpu().numpy(), s_ref) < STATE_REL


@pytest.mark.parametrize("tag", list(inputs.GDN_CASES))
def test_gdn_scan_on_reference_layer_inputs(cuda, tag):
    """The reference layer's own scan (golden, pre out_proj) from the kernels."""
    from hybrid_llm_b200 import kernels
    g = golden("gdn")
    c = inputs.gdn_case(tag)
    p, x = c["p"], c["hidden"].astype(np.float64)
    b, t, _ = x.shape
    h, kd, vd = c["heads"], c["key_dim"], c["value_dim"]
    proj = np.concatenate([x @ p["q_proj"].T, x @ p["k_proj"].T, x @ p["v_proj"].T,
                           x @ p["gate_proj"].T, x @ p["beta_proj"].T], axis=-1)
    pad = (-proj.shape[-1]) % 8  # the fused projection is padded to 16-byte rows
    proj = np.concatenate([proj, np.zeros(proj.shape[:-1] + (pad,))], axis=-1)
    pr = _bf(proj.reshape(b * t, -1)).cuda()
    kernels.gdn_activate(pr, h, kd, vd, torch.from_numpy(p["beta_bias"]).cuda())
    pr = pr.view(b, t, -1)
    hk, hv = h * kd, h * vd
    q = pr[..., :hk].unflatten(-1, (h, kd))
    k = pr[..., hk:2 * hk].unflatten(-1, (h, kd))
    v = pr[..., 2 * hk:2 * hk + hv].unflatten(-1, (h, vd))
    gate = pr[..., 2 * hk + hv:2 * hk + 2 * hv].unflatten(-1, (h, vd))
    beta = pr[..., 2 * hk + 2 * hv:2 * hk + 2 * hv + h]
    st = torch.from_numpy(c["state"]).cuda()
    out = kernels.gdn_prefill(q, k, v, gate, beta, st,
                              decay_logit=torch.from_numpy(p["decay_logit"]).cuda(),
                              reset=torch.from_numpy(c["reset"]).cuda())
    torch.cuda.synchronize()
    assert _rel(_f(out).reshape(b, t, -1), g[f"{tag}_scan"]) < 3 * OUT_REL
    assert _rel(st.cpu().numpy(), g[f"{tag}_prefill_state"]) < 3e-2


@pytest.mark.parametrize("t,hist", [(37, False), (1, True), (5, True)])
def test_conv_gate_matches_oracle(cuda, t, hist):
    from hybrid_llm_b200 import kernels
    rng = np.random.default_rng(t)
    b, d = 3, 256
    x = _bf(rng.normal(size=(b, t, d)))
    y = _bf(rng.normal(size=(b, t, d)))
    w = rng.normal(0, 0.3, (d, 1, 4)).astype(np.float32)
    reset = np.zeros((b, t), bool)
    if t > 3:
        reset[1, 2] = True
    reset[2, 0] = True
    history = _bf(rng.normal(size=(b, 3, d))) if hist else None
    res = _bf(rng.normal(size=(b, t, d)))
    got = kernels.gdn_conv_gate(x.cuda(), y.cuda(), torch.from_numpy(w).cuda(),
                                history=None if history is None else history.clone().cuda(),
                                reset=torch.from_numpy(reset).cuda(), residual=res.clone().cuda())
    torch.cuda.synchronize()
    conv = gdn.causal_conv(_f(x), w, reset, None if history is None else _f(history))
    ref = _f(res) + _f(y) * gdn.sigmoid(conv)
    assert _rel(_f(got), ref) < 1e-2


def test_conv_history_roll(cuda):
    from hybrid_llm_b200 import kernels
    rng = np.random.default_rng(1)
    b, d = 2, 128
    history = _bf(rng.normal(size=(b, 3, d))).cuda()
    old = history.clone()
    x = _bf(rng.normal(size=(b, 1, d))).cuda()
    kernels.gdn_conv_gate(x, x, torch.zeros(d, 4, device="cuda"), history=history,
                          out=torch.empty_like(x), roll_history=True)
    torch.cuda.synchronize()
    assert torch.equal(history[:, :2], old[:, 1:]) and torch.equal(history[:, 2:], x)


def test_gdn_step_raw_inputs_equal_activated_inputs(cuda):
    """llmyb_gdn_step with raw projections (in-kernel activation) = activate + step."""
    from hybrid_llm_b200 import kernels
    rng = np.random.default_rng(5)
    b, h, kd, vd = 3, 4, 128, 64
    width = 2 * h * (kd + vd) + h
    width += (-width) % 8
    proj = _bf(rng.normal(0, 1, (b, width))).cuda()
    bias = torch.from_numpy(rng.normal(0, 0.5, h).astype(np.float32)).cuda()
    dl = torch.from_numpy(rng.uniform(0.5, 3, h).astype(np.float32)).cuda()
    st0 = torch.from_numpy(rng.normal(0, 0.3, (b, h, kd, vd)).astype(np.float32)).cuda()

    def views(pr):
        hk, hv = h * kd, h * vd
        return (pr[:, :hk].unflatten(-1, (h, kd)), pr[:, hk:2 * hk].unflatten(-1, (h, kd)),
                pr[:, 2 * hk:2 * hk + hv].unflatten(-1, (h, vd)),
                pr[:, 2 * hk + hv:2 * hk + 2 * hv].unflatten(-1, (h, vd)),
                pr[:, 2 * hk + 2 * hv:2 * hk + 2 * hv + h])

    s_raw = st0.clone()
    o_raw = kernels.gdn_step(*views(proj), s_raw, decay_logit=dl, raw_inputs=True, beta_bias=bias)
    act = proj.clone()
    kernels.gdn_activate(act, h, kd, vd, bias)
    s_act = st0.clone()
    o_act = kernels.gdn_step(*views(act), s_act, decay_logit=dl)
    torch.cuda.synchronize()
    assert _rel(_f(o_raw), _f(o_act)) < 2e-2
    assert _rel(s_raw.cpu().numpy(), s_act.cpu().numpy()) < 1e-2


def _torch_conv_gate(x, y, w, reset, residual=None):
    """fp32 torch restatement of the prompt conv gate: tap x[t - s] (s = 3..0)
    is kept when it exists and no reset lies in (t - s, t]."""
    xf, yf = x.float(), y.float()
    b, t, d = xf.shape
    seg = torch.cumsum(reset.int(), dim=1)
    acc = torch.zeros_like(xf)
    for j in range(4):
        s = 3 - j
        xs = torch.zeros_like(xf)
        ok = torch.zeros(b, t, dtype=torch.bool, device=x.device)
        if s < t:
            xs[:, s:] = xf[:, :t - s]
            ok[:, s:] = seg[:, :t - s] == seg[:, s:]
        acc += w[:, j].float() * xs * ok[..., None]
    out = (yf * torch.sigmoid(acc)).bfloat16().float()
    return out if residual is None else residual.float() + out


@pytest.mark.parametrize("b,t,d", [(3, 100, 256), (4, 4096, 512), (8, 4096, 2048)])
@pytest.mark.parametrize("add", [False, True])
def test_conv_gate_prompt_runs_match_torch(cuda, b, t, d, add):
    """The run kernel of the prompt conv gate (each thread slides the taps over
    1 to 16 tokens; the three sizes select runs of 1, 2 and 16) with resets at
    run boundaries, inside runs and at token 0."""
    from hybrid_llm_b200 import kernels
    g = torch.Generator(device="cuda").manual_seed(b * t + d)
    x = torch.randn(b, t, d, device="cuda", generator=g).bfloat16()
    y = torch.randn(b, t, d, device="cuda", generator=g).bfloat16()
    w = torch.randn(d, 4, device="cuda", generator=g) * 0.3
    reset = torch.zeros(b, t, dtype=torch.bool, device="cuda")
    for p in (0, 1, 15, 16, 17, 31, 33, 34, t - 1):
        reset[p % b, min(p, t - 1)] = True
    reset[:, :: 97] |= torch.rand(b, (t + 96) // 97, device="cuda", generator=g) < 0.5
    res = torch.randn(b, t, d, device="cuda", generator=g).bfloat16() if add else None
    got = kernels.gdn_conv_gate(x, y, w, reset=reset,
                                residual=None if res is None else res.clone())
    kernels.check_device_status()
    ref = _torch_conv_gate(x, y, w, reset, res)
    err = (got.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-2, err


@pytest.mark.parametrize("h,kd,vd", [(12, 64, 64), (16, 128, 128), (4, 128, 64)])
def test_gdn_activate_vector_path_matches_reference(cuda, h, kd, vd):
    """16-byte rows (the model's padded projection) take the piece-per-thread
    kernel, other widths the per-head warp kernel; both against fp64."""
    from hybrid_llm_b200 import kernels
    n = 300
    base = 2 * h * (kd + vd) + h
    g = torch.Generator(device="cuda").manual_seed(h + kd)
    bias = torch.randn(h, device="cuda", generator=g)
    for width in (base + (-base) % 8, base + (1 if (base + 1) % 8 else 2)):
        proj = (torch.randn(n, width, device="cuda", generator=g) * 2).bfloat16()
        ref = proj.double().clone()
        kernels.gdn_activate(proj, h, kd, vd, bias)
        kernels.check_device_status()
        hk, hv = h * kd, h * vd
        qk = ref[:, :2 * hk].view(n, 2 * h, kd)
        ref[:, :2 * hk] = (qk / qk.square().sum(-1, keepdim=True).clamp_min(1e-12).sqrt()).view(n, -1)
        ref[:, 2 * hk + hv:2 * hk + 2 * hv] = torch.sigmoid(ref[:, 2 * hk + hv:2 * hk + 2 * hv])
        ref[:, 2 * hk + 2 * hv:2 * hk + 2 * hv + h] = torch.sigmoid(
            ref[:, 2 * hk + 2 * hv:2 * hk + 2 * hv + h] + bias.double())
        err = (proj.double() - ref).abs().max().item()
        assert err < 8e-3, (width, err)
