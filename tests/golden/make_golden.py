"""Generate the golden fixtures by running the reference's own PyTorch code.

Run in a container that has the reference checkout (``LLMY_REFERENCE``;
by default the directory ``reference`` beside this repository)::

    python tests/golden/make_golden.py [section ...]

Each section seeds its inputs with numpy, runs the reference modules on CPU
(fp32, Triton off) and writes ``tests/golden/<section>.npz``.  The fixtures
are small; the tests compare the numpy oracle against them on CPU and the CUDA
kernels against the oracle on a GPU.  Nothing at run time reads the reference.
"""
from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("LLMY_REFERENCE",
                        Path(__file__).resolve().parents[2].parent / "reference"))
sys.path.insert(0, str(HERE.parents[1]))  # repo root, for the weight generator

os.environ.setdefault("LLMY_DISABLE_TRITON", "1")

import torch  # noqa: E402

sys.path.insert(0, str(HERE))
import inputs  # noqa: E402

torch.set_num_threads(max(1, os.cpu_count() or 1))


def _ref_import():
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import model.layers.gated_deltanet as gdn_mod  # noqa: F401
    import model.layers.moe as moe_mod
    gdn_mod._triton_gdn_available = False
    moe_mod._triton_available = False
    return gdn_mod, moe_mod


def _standalone():
    """Import sample_standalone.py as a module (it must be in sys.modules first)."""
    name = "llmy_sample_standalone"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, REF / "sample_standalone.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def save(name: str, **arrays) -> None:
    path = HERE / f"{name}.npz"
    np.savez_compressed(path, **{k: np.asarray(v) for k, v in arrays.items()})
    print(f"wrote {path.relative_to(HERE.parents[1])} ({path.stat().st_size} bytes)")


def t(x) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x))


# ----------------------------------------------------------------- sections
def sec_router() -> None:
    """ContextAwareRouter.forward (context_router.py:59-86), context off."""
    _ref_import()
    from model.layers.context_router import ContextAwareRouter

    out = {}
    for tag in inputs.ROUTER_CASES:
        c = inputs.router_case(tag)
        n, d = c["hidden"].shape[1:]
        e, k = c["weight"].shape[0], c["k"]
        router = ContextAwareRouter(d, e, k, context_aware=False)
        with torch.no_grad():
            router.logits.weight.copy_(t(c["weight"]))
        captured = {}
        router.logits.register_forward_hook(lambda m, i, o: captured.setdefault("logits", o.detach()))
        with torch.no_grad():
            idx, prob, _ = router(t(c["hidden"]), return_stats=False)
        flat = idx.reshape(-1)
        _, stable = torch.sort(flat, stable=True)
        _, unstable = torch.sort(flat)
        out.update({
            f"{tag}_checksum": inputs.checksum(c["hidden"], c["weight"]),
            f"{tag}_logits": captured["logits"].reshape(n, e).numpy(),
            f"{tag}_idx": idx.reshape(n, k).numpy(), f"{tag}_prob": prob.reshape(n, k).numpy(),
            f"{tag}_stable_order": stable.numpy(), f"{tag}_unstable_order": unstable.numpy(),
            f"{tag}_counts": torch.bincount(flat, minlength=e).numpy(),
        })
    save("router", **out)


def sec_moe() -> None:
    """_moe_dispatch_fused (moe.py:29-82) with torch.topk routes, fp32."""
    _, moe_mod = _ref_import()
    out = {}
    for tag in inputs.MOE_CASES:
        c = inputs.moe_case(tag)
        vals, idx = torch.topk(t(c["logits"]), c["k"], dim=-1)
        prob = vals.softmax(-1)
        with torch.no_grad():
            y = moe_mod._moe_dispatch_fused(t(c["flat"]), idx, prob, t(c["w_gate"]),
                                            t(c["w_up"]), t(c["w_down"]))
        out.update({f"{tag}_checksum": inputs.checksum(*(c[k] for k in ("flat", "logits", "w_gate", "w_up", "w_down"))),
                    f"{tag}_idx": idx.numpy(), f"{tag}_prob": prob.numpy(), f"{tag}_out": y.numpy()})
    save("moe", **out)


def sec_gdn() -> None:
    """GatedDeltaNet.forward (gated_deltanet.py:119-276): prefill with resets, then
    three decode steps with the conv history the block keeps (model/model.py:283-289)."""
    gdn_mod, _ = _ref_import()
    out = {}
    for tag in inputs.GDN_CASES:
        c = inputs.gdn_case(tag)
        p = c["p"]
        d = c["hidden"].shape[-1]
        m = gdn_mod.GatedDeltaNet(d, c["heads"], c["heads"], c["key_dim"], c["value_dim"], 4)
        with torch.no_grad():
            for name in ("q_proj", "k_proj", "v_proj", "beta_proj", "gate_proj", "out_proj"):
                getattr(m, name).weight.copy_(t(p[name]))
            m.beta_proj.bias.copy_(t(p["beta_bias"]))
            m.conv.weight.copy_(t(p["conv"]))
            m.decay_logit.copy_(t(p["decay_logit"]))
        scan = []
        m.out_proj.register_forward_pre_hook(lambda mod, a: scan.append(a[0].detach().clone()))
        with torch.no_grad():
            y, s_pre = m(t(c["hidden"]), t(c["state"]), t(c["reset"]), reference=True)
            s = s_pre.clone()
            hist = t(c["hidden"])[:, -3:].clone()
            ys, ss = [], []
            for i in range(c["steps"].shape[1]):
                x1 = t(c["steps"][:, i:i + 1])
                y1, s = m(x1, s.clone(), None, conv_history=hist)
                hist = torch.cat([hist[:, 1:], x1], dim=1)
                ys.append(y1.numpy())
                ss.append(s.numpy())
        out.update({f"{tag}_checksum": inputs.checksum(c["hidden"], c["state"], *p.values()),
                    f"{tag}_out": y.numpy(), f"{tag}_prefill_state": s_pre.numpy(),
                    f"{tag}_scan": scan[0].numpy(), f"{tag}_step_out": np.stack(ys, 1),
                    f"{tag}_step_state": ss[-1]})
    save("gdn", **out)


def sec_csa() -> None:
    """CompressedSelectiveAttention (csa.py:35-259) with the remote branch
    disabled (temporal_compression=10**9): prefill, then decode steps that
    keep the normed-hidden local history as PhysicalBlock does
    (model/model.py:340-357)."""
    _ref_import()
    from model.layers.csa import CompressedSelectiveAttention

    out = {}
    for tag in inputs.CSA_CASES:
        c = inputs.csa_case(tag)
        d = c["hidden"].shape[-1]
        m = CompressedSelectiveAttention(d, compression=10**9, local_window=c["window"],
                                         index_heads=c["heads"], index_head_dim=c["head_dim"],
                                         top_k=4)
        with torch.no_grad():
            for name, w in c["p"].items():
                getattr(m, name).weight.copy_(t(w))
            y, _, _ = m(t(c["hidden"]), return_stats=False)
            hist = t(c["hidden"])[:, -(c["window"] - 1):].clone()
            ys = []
            for i in range(c["steps"].shape[1]):
                x1 = t(c["steps"][:, i:i + 1])
                valid = torch.ones(hist.shape[:2], dtype=torch.bool)
                y1, _, _ = m.forward_step(x1, local_history=hist, local_history_valid=valid,
                                          position=torch.full((x1.shape[0],), c["hidden"].shape[1] + i))
                hist = torch.cat([hist, x1], dim=1)[:, -(c["window"] - 1):]
                ys.append(y1.numpy())
        out.update({f"{tag}_checksum": inputs.checksum(c["hidden"], *c["p"].values()),
                    f"{tag}_out": y.numpy(), f"{tag}_step_out": np.stack(ys, 1)})
    save("csa", **out)


def sec_band() -> None:
    """fused_banded_local_attention (sample_standalone.py:70-85), per-head V."""
    sa = _standalone()
    out = {}
    for tag in inputs.BAND_CASES:
        c = inputs.band_case(tag)
        with torch.no_grad():
            y = sa.fused_banded_local_attention(t(c["q"]), t(c["k"]), t(c["v"]),
                                                window_size=c["window"])
        out.update({f"{tag}_checksum": inputs.checksum(c["q"], c["k"], c["v"]),
                    f"{tag}_out": y.numpy()})
    save("band", **out)


def sec_sample() -> None:
    """_sample_next_token (sample_standalone.py:5383-5423), one row at a time, with
    torch.multinomial replaced by the deterministic inverse CDF on a given uniform."""
    sa = _standalone()
    out = {}
    real_multinomial = torch.multinomial
    for tag in inputs.SAMPLE_CASES:
        c = inputs.sample_case(tag)
        toks, lps, kept = [], [], []
        for r in range(c["logits"].shape[0]):
            u = float(c["uniforms"][r])
            seen_probs = []

            def fake_multinomial(probs, n, *a, **k):
                pr = probs.double()
                cum = torch.cumsum(pr, dim=-1)
                hit = torch.nonzero(u < cum[0])
                idx = int(hit[0, 0]) if hit.numel() else int(torch.nonzero(pr[0] > 0)[-1, 0])
                seen_probs.append(probs[0].clone())
                return torch.tensor([[idx]])

            torch.multinomial = fake_multinomial
            try:
                tok, lp = sa._sample_next_token(t(c["logits"][r:r + 1]), c["generated"][r],
                                                temp=c["temp"], top_k=c["top_k"], top_p=c["top_p"],
                                                rep=c["rep"])
            finally:
                torch.multinomial = real_multinomial
            toks.append(int(tok))
            lps.append(float(lp))
            kept.append(float(seen_probs[0].max()) if seen_probs else 1.0)
        out.update({f"{tag}_checksum": inputs.checksum(c["logits"], c["uniforms"]),
                    f"{tag}_tokens": np.array(toks), f"{tag}_logprob": np.array(lps),
                    f"{tag}_max_prob": np.array(kept)})
    save("sample", **out)


def _reference_model(cfg, standalone: bool = False):
    """The reference model with the synthetic weights.  standalone=True builds
    the copy in sample_standalone.py, whose decode_step carries the loop
    output (model/model.py:846-905 leaves `streams` unchanged when every row
    is active, so its decode logits skip the recurrent core)."""
    from hybrid_llm_b200.weights import synthetic_state_dict

    if standalone:
        sa = _standalone()
        V6Config, LoopedHybridMoEForCausalLM = sa.V6Config, sa.LoopedHybridMoEForCausalLM
    else:
        _ref_import()
        from model.config import V6Config
        from model.model import LoopedHybridMoEForCausalLM

    model = LoopedHybridMoEForCausalLM(V6Config.from_mapping(inputs.v6_mapping(cfg))).eval()
    sd = synthetic_state_dict(cfg, seed=0)
    own = dict(model.named_parameters())
    with torch.no_grad():
        for name in sd:
            own[name].copy_(sd[name].reshape(own[name].shape))
    return model


def sec_model() -> None:
    """LoopedHybridMoEForCausalLM.forward + 6 greedy decode_step calls on the mini
    config, and the single looped block on hidden states [1, 256, 512]."""
    from hybrid_llm_b200.config import single_block_config

    _ref_import()
    from model.recurrent_state import RecurrentState

    cfg = inputs.mini_config()
    model = _reference_model(cfg, standalone=True)
    ids = torch.from_numpy(inputs.mini_prompt())
    with torch.no_grad():
        out = model(ids, collect_diagnostics=False)
        state = out.state
        logits = out.logits[:, -1]
        toks, step_logits = [], []
        for _ in range(6):
            nxt = logits.argmax(-1, keepdim=True)
            toks.append(nxt[:, 0].numpy())
            o = model.decode_step(nxt, state=state)
            logits = o.logits[:, -1]
            step_logits.append(logits.numpy())
    res = {"mini_prefill_last": out.logits[:, -1].numpy(), "mini_tokens": np.stack(toks, 1),
           "mini_step_logits": np.stack(step_logits, 1)}
    # model/model.py's decode_step on the same inputs (loop output dropped)
    pkg = _reference_model(cfg)
    with torch.no_grad():
        o1 = pkg(ids, collect_diagnostics=False)
        o2 = pkg.decode_step(o1.logits[:, -1].argmax(-1, keepdim=True), state=o1.state)
    res["mini_pkg_prefill_last"] = o1.logits[:, -1].numpy()
    res["mini_pkg_step0_logits"] = o2.logits[:, -1].numpy()

    bcfg = single_block_config()
    bmodel = _reference_model(bcfg)
    x = torch.from_numpy(inputs.block_hidden())
    with torch.no_grad():
        st = RecurrentState()
        streams = x.unsqueeze(-2)
        for i in range(bcfg.num_loops):
            streams, _ = bmodel._run_stack(bmodel.recurrent_core, streams, st, segment_ids=None,
                                           reset_mask=None, diagnostics={},
                                           collect_diagnostics=False, state_namespace=f"loop{i}")
    res["block_out_rows"] = streams[0, ::4, 0].numpy()
    res["block_checksum"] = inputs.checksum(inputs.block_hidden())
    save("model", **res)


def _prefill_and_decode(cfg, tag: str, steps: int = 4) -> dict:
    """Prefill logits of the package model and of sample_standalone.py's copy,
    then greedy decode from the standalone copy (the loop output carried)."""
    ids = torch.from_numpy(inputs.mini_prompt())
    pkg = _reference_model(cfg)
    sa = _reference_model(cfg, standalone=True)
    res = {}
    with torch.no_grad():
        res[f"{tag}_prefill_last"] = pkg(ids, collect_diagnostics=False).logits[:, -1].numpy()
        out = sa(ids, collect_diagnostics=False)
        res[f"{tag}_sa_prefill_last"] = out.logits[:, -1].numpy()
        state, logits = out.state, out.logits[:, -1]
        toks, step_logits = [], []
        for _ in range(steps):
            nxt = logits.argmax(-1, keepdim=True)
            toks.append(nxt[:, 0].numpy())
            logits = sa.decode_step(nxt, state=state).logits[:, -1]
            step_logits.append(logits.numpy())
    res[f"{tag}_tokens"] = np.stack(toks, 1)
    res[f"{tag}_step_logits"] = np.stack(step_logits, 1)
    return res


def sec_combined() -> None:
    """mHC, router context, CSA remote branch and shared experts together."""
    save("combined", **_prefill_and_decode(inputs.combined_config(), "cb", steps=6))


def sec_loop_mem() -> None:
    """The mini model with the loop memory (loop_memory.py) between its three loops."""
    save("loop_mem", **_prefill_and_decode(inputs.loop_memory_config(), "lm", steps=4))


def sec_shared() -> None:
    """The mini model with two shared experts next to the routed ones."""
    save("shared", **_prefill_and_decode(inputs.shared_experts_config(), "sh", steps=4))


def sec_csa_remote() -> None:
    """The mini model with the CSA remote compressed branch (4-token summaries,
    top-3); eight decode steps complete two more summaries."""
    save("csa_remote", **_prefill_and_decode(inputs.csa_remote_config(), "cr", steps=8))


def sec_router_ctx() -> None:
    """The mini model with the context-aware router (64-wide latents, window 8)."""
    save("router_ctx", **_prefill_and_decode(inputs.router_ctx_config(), "rc", steps=10))


def sec_mhc() -> None:
    """The mini model with four hyper-connection streams: prefill logits of the
    package model, and greedy decode from sample_standalone.py's copy (the
    loop output carried, as for the mini model above)."""
    cfg = inputs.mhc_config()
    ids = torch.from_numpy(inputs.mini_prompt())
    pkg = _reference_model(cfg)
    sa = _reference_model(cfg, standalone=True)
    res = {}
    with torch.no_grad():
        o1 = pkg(ids, collect_diagnostics=False)
        res["mhc_prefill_last"] = o1.logits[:, -1].numpy()
        out = sa(ids, collect_diagnostics=False)
        res["mhc_sa_prefill_last"] = out.logits[:, -1].numpy()
        state, logits = out.state, out.logits[:, -1]
        toks, step_logits = [], []
        for _ in range(4):
            nxt = logits.argmax(-1, keepdim=True)
            toks.append(nxt[:, 0].numpy())
            o = sa.decode_step(nxt, state=state)
            logits = o.logits[:, -1]
            step_logits.append(logits.numpy())
    res["mhc_tokens"] = np.stack(toks, 1)
    res["mhc_step_logits"] = np.stack(step_logits, 1)
    save("mhc", **res)


SECTIONS = {"loop_mem": sec_loop_mem, "combined": sec_combined, "shared": sec_shared, "csa_remote": sec_csa_remote, "router_ctx": sec_router_ctx, "mhc": sec_mhc, "model": sec_model, "sample": sec_sample, "router": sec_router, "moe": sec_moe, "gdn": sec_gdn, "csa": sec_csa, "band": sec_band}


def main(argv: list[str]) -> None:
    if not REF.exists():
        raise SystemExit(f"reference checkout not found at {REF}")
    names = argv or list(SECTIONS)
    for name in names:
        SECTIONS[name]()


if __name__ == "__main__":
    main(sys.argv[1:])
