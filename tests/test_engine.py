"""The reference engine's API (llmy_cuda/include/llmy.h) over this build.

Host sampler: the numpy restatement (oracle/sampling.py) and the native
llmyb_engine_sample are pinned to golden vectors made by the reference's own
llmy_sample (tests/golden/make_llmy_sample.py).  Engine calls on the GPU are
checked against the model they wrap: bit-identical logits."""
import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from hybrid_llm_b200 import engine
from oracle import sampling

GOLDEN = Path(__file__).resolve().parent / "golden"


def _cases():
    z = np.load(GOLDEN / "llmy_sample.npz")
    for i in range(z["token"].size):
        v, lo = int(z["vocab"][i]), int(z["logit_off"][i])
        ro, nr = int(z["recent_off"][i]), int(z["n_recent"][i])
        yield dict(logits=z["logits"][lo:lo + v], vocab=v, temperature=float(z["temperature"][i]),
                   top_k=int(z["top_k"][i]), top_p=float(z["top_p"][i]), rep=float(z["rep"][i]),
                   recent=z["recent"][ro:ro + nr], state_in=int(z["state_in"][i]),
                   state_out=int(z["state_out"][i]), token=int(z["token"][i]))


def test_golden_cover_the_sampler_rules():
    cases = list(_cases())
    assert len(cases) == 96
    assert {c["temperature"] > 0 for c in cases} == {True, False}
    assert any(c["top_k"] > 256 for c in cases) and any(0 < c["top_p"] < 1 for c in cases)
    assert any(c["rep"] != 1 and len(c["recent"]) for c in cases)
    assert max(c["vocab"] for c in cases) == 32000 and min(c["vocab"] for c in cases) == 1


def test_oracle_matches_reference_sampler():
    for c in _cases():
        tok, st = sampling.engine_host_sample(c["logits"], c["temperature"], c["top_k"], c["top_p"],
                                              c["rep"], c["recent"], c["state_in"])
        assert (tok, st) == (c["token"], c["state_out"]), c


def test_native_sampler_matches_reference_sampler():
    for c in _cases():
        st = np.array([c["state_in"]], dtype=np.uint64)
        tok = engine.llmy_sample(c["logits"], c["vocab"], c["temperature"], c["top_k"], c["top_p"],
                                 c["rep"], c["recent"], len(c["recent"]), st)
        assert (tok, int(st[0])) == (c["token"], c["state_out"]), c


def test_sampler_argument_forms():
    rng = np.random.default_rng(7)
    lg = rng.normal(size=500).astype(np.float32)
    # greedy: argmax, state untouched
    st = ctypes.c_uint64(99)
    assert engine.llmy_sample(lg, 500, 0.0, 0, 1.0, 1.0, None, 0, st) == int(lg.argmax())
    assert st.value == 99
    # a torch tensor and a ctypes array give the same draw as numpy
    toks = []
    for logits in (lg, torch.from_numpy(lg.copy()), (ctypes.c_float * 500)(*lg.tolist())):
        s = ctypes.c_uint64(12345)
        toks.append((engine.llmy_sample(logits, 500, 0.9, 40, 0.9, 1.2, [3, 3, 7], 3, s), s.value))
    assert toks[0] == toks[1] == toks[2]
    assert toks[0] == sampling.engine_host_sample(lg, 0.9, 40, 0.9, 1.2, [3, 3, 7], 12345)
    assert engine.llmy_sample(lg, 0, 1.0, 0, 1.0, 1.0, None, 0, ctypes.c_uint64(1)) == 0
    with pytest.raises(TypeError):
        engine.llmy_sample(lg, 500, 1.0, 0, 1.0, 1.0, None, 0, 5)


def test_load_failure_returns_none(tmp_path, capsys):
    assert engine.llmy_load(tmp_path / "missing.llmy") is None
    bad = tmp_path / "bad.llmy"
    bad.write_bytes(b"GGUF" + bytes(64))
    assert engine.llmy_load(str(bad)) is None
    err = capsys.readouterr().err
    assert err.count("[llmy_load]") == 2


@pytest.mark.gpu
def test_engine_prefill_decode_equal_the_model(cuda):
    """llmy_prefill / llmy_decode on the converter's fixture give the wrapped
    model's logits bit for bit, into host, device and ctypes buffers."""
    import inputs
    from hybrid_llm_b200.state import RecurrentState

    m = engine.llmy_load(GOLDEN / "tiny_model.llmy")
    assert m is not None
    cfg = inputs.llmy_config()
    assert (engine.llmy_vocab_size(m), engine.llmy_d_model(m)) == (cfg.vocab_size, cfg.d_model)
    assert engine.llmy_num_loops(m) == engine.llmy_max_loops(m) == cfg.num_loops
    assert engine.llmy_mhc_streams(m) == 1
    v = cfg.vocab_size
    prompt = np.random.default_rng(5).integers(0, v, size=37).astype(np.int32)

    s = engine.llmy_state_new(m)
    host = np.zeros(v, dtype=np.float32)
    engine.llmy_prefill(m, s, prompt, prompt.size, host)
    assert engine.llmy_last_executed_loops(s) == cfg.num_loops

    st = RecurrentState(cfg, 1, cuda)
    ref = m.model.forward(torch.from_numpy(prompt.astype(np.int64))[None].to(cuda), state=st,
                          last_logits_only=True)
    assert np.array_equal(host, ref.logits[0, -1].float().cpu().numpy())

    tok = int(host.argmax())
    dev = torch.zeros(v, dtype=torch.float32, device=cuda)
    cbuf = (ctypes.c_float * v)()
    for step in range(3):
        pos = prompt.size + step
        out = dev if step == 0 else (cbuf if step == 1 else host)
        engine.llmy_decode(m, s, tok, pos, 0, out)
        want = m.model.decode_step(torch.tensor([tok], device=cuda), st)[0].float().cpu().numpy()
        got = out.cpu().numpy() if isinstance(out, torch.Tensor) else np.ctypeslib.as_array(out)
        assert np.array_equal(got, want), step
        tok = int(np.argmax(got))

    # fewer loops for one step: the model's decode with the same loop count
    st_copy = RecurrentState(cfg, 1, cuda)
    st_copy.load_state_dict(st.state_dict())
    engine.llmy_decode(m, s, tok, prompt.size + 3, 1, host)
    assert engine.llmy_last_executed_loops(s) == 1
    want = m.model.decode_step(torch.tensor([tok], device=cuda), st_copy, num_loops=1)
    assert np.array_equal(host, want[0].float().cpu().numpy())

    # a reset state replays the prompt to the same logits
    first = host.copy()
    engine.llmy_state_reset(s)
    again = np.zeros(v, dtype=np.float32)
    engine.llmy_prefill(m, s, prompt, prompt.size, again)
    s2 = engine.llmy_state_new(m)
    fresh = np.zeros(v, dtype=np.float32)
    engine.llmy_prefill(m, s2, prompt, prompt.size, fresh)
    assert np.array_equal(again, fresh) and not np.array_equal(again, first)
    engine.llmy_state_free(s)
    engine.llmy_state_free(s2)
    engine.llmy_free(m)


@pytest.mark.gpu
def test_engine_generation_loop(cuda):
    """The reference sampler loop (prefill, sample, decode at increasing
    positions) with greedy sampling reproduces the model's greedy decode."""
    m = engine.llmy_load(GOLDEN / "tiny_model.llmy")
    v = engine.llmy_vocab_size(m)
    prompt = np.arange(11, dtype=np.int32) * 7 % v
    s = engine.llmy_state_new(m)
    logits = np.zeros(v, dtype=np.float32)
    engine.llmy_prefill(m, s, prompt, prompt.size, logits)
    rng = ctypes.c_uint64(1)
    toks = []
    for step in range(5):
        tok = engine.llmy_sample(logits, v, 0.0, 0, 1.0, 1.0, None, 0, rng)
        toks.append(tok)
        engine.llmy_decode(m, s, tok, prompt.size + step, 0, logits)
    out = m.model.forward(torch.from_numpy(prompt.astype(np.int64))[None].to(cuda),
                          last_logits_only=True)
    st, nxt, ref = out.state, int(out.logits[0, -1].float().argmax()), []
    for _ in range(5):
        ref.append(nxt)
        nxt = int(m.model.decode_step(torch.tensor([nxt], device=cuda), st)[0].float().argmax())
    assert toks == ref


# ------------------------------------------------ engine device entry points
def _ops():
    return np.load(GOLDEN / "engine_ops.npz")


def test_sinkhorn_oracle_matches_reference():
    from oracle import mhc
    z = _ops()
    for it in (0, 1, 5, 20):
        want = z[f"sk_out_{it}"]
        got = mhc.sinkhorn(z["sk_in"], it)
        assert np.allclose(got, want, rtol=2e-6, atol=1e-6), it
    # the last step normalises columns: each column sums to one
    s = mhc.sinkhorn(z["sk_in"], 20)
    assert np.allclose(s.sum(-2), 1, atol=1e-6)


def test_moe_selected_oracle_matches_reference():
    from oracle import routing
    z = _ops()
    gu = z["moe_gate_up"]
    h = gu.shape[1] // 2
    got = routing.moe_forward(z["moe_x"][None], z["moe_idx"][None], z["moe_prob"][None],
                              gu[:, :h], gu[:, h:], z["moe_down"])[0]
    assert np.allclose(got, z["moe_out"], rtol=1e-5, atol=1e-6)


@pytest.mark.gpu
def test_sinkhorn4_kernel(cuda):
    """fp32 tolerance: accurate expf/logf in a different summation order than
    torch.logsumexp (rtol 2e-6 on the golden, 1e-5 on a large random batch)."""
    from hybrid_llm_b200 import kernels
    from oracle import mhc
    z = _ops()
    x = torch.from_numpy(z["sk_in"]).to(cuda)
    for it in (0, 1, 5, 20):
        got = kernels.mhc_sinkhorn4(x, it).cpu().numpy()
        assert np.allclose(got, z[f"sk_out_{it}"], rtol=2e-6, atol=1e-6), it
    big = torch.randn(3, 1000, 4, 4, device=cuda) * 3
    got = kernels.mhc_sinkhorn4(big, 20).cpu().numpy()
    assert np.allclose(got, mhc.sinkhorn(big.cpu().numpy(), 20), rtol=1e-5, atol=1e-6)
    # the engine-ABI form: raw buffers, status codes
    out = torch.empty_like(x)
    assert engine.llmy_mhc_sinkhorn4(x, out, x.shape[0], 20) == 0
    assert np.allclose(out.cpu().numpy(), z["sk_out_20"], rtol=2e-6, atol=1e-6)
    assert engine.llmy_mhc_sinkhorn4(x, out, 0, 20) == 1
    assert engine.llmy_mhc_sinkhorn4(x, out, 4, -1) == 1
    assert engine.llmy_mhc_sinkhorn4(None, out, 4, 3) == 1
    torch.cuda.synchronize()


@pytest.mark.gpu
def test_moe_selected_fp32_kernel(cuda):
    from hybrid_llm_b200 import kernels
    from oracle import routing
    z = _ops()
    t = {k: torch.from_numpy(np.ascontiguousarray(z[k])).to(cuda)
         for k in ("moe_x", "moe_idx", "moe_prob", "moe_gate_up", "moe_down")}
    got = kernels.moe_selected_fp32(t["moe_x"], t["moe_idx"], t["moe_prob"], t["moe_gate_up"],
                                    t["moe_down"]).cpu().numpy()
    assert np.allclose(got, z["moe_out"], rtol=1e-5, atol=1e-6)
    # an odd width (scalar loads), an expert id outside [0, E) contributes zero
    rng = np.random.default_rng(3)
    e, d, h = 5, 37, 23
    x = rng.normal(size=d).astype(np.float32)
    gu = (rng.normal(size=(e, 2 * h, d)) * 0.2).astype(np.float32)
    dn = (rng.normal(size=(e, d, h)) * 0.2).astype(np.float32)
    idx = np.array([4, -1, 1, 7], dtype=np.int64)
    prob = np.array([0.4, 0.3, 0.2, 0.1], dtype=np.float32)
    act = torch.empty(4, h, device=cuda)
    route = torch.empty(4, d, device=cuda)
    out = torch.empty(d, device=cuda)
    dev = [torch.from_numpy(a).to(cuda) for a in (x, idx, prob, gu, dn)]
    assert engine.llmy_moe_selected_fp32(*dev, act, route, out, d, h, e, 4) == 0
    keep = idx[[0, 2]]
    want = routing.moe_forward(x[None], keep[None], prob[[0, 2]][None], gu[:, :h], gu[:, h:], dn)[0]
    assert np.allclose(out.cpu().numpy(), want, rtol=1e-5, atol=1e-6)
    r = route.cpu().numpy()
    assert not r[1].any() and not r[3].any()
    assert np.array_equal(out.cpu().numpy(), ((r[0] + r[1]) + r[2]) + r[3])
    assert engine.llmy_moe_selected_fp32(*dev, act, route, out, d, h, e, 0) == 1
    torch.cuda.synchronize()
