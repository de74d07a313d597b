"""Seeded inputs shared by the golden generator and the tests.

The fixtures store only the reference's outputs (plus a checksum of the
inputs); both sides rebuild the inputs from these functions, so the committed
files stay small.
"""
from __future__ import annotations

import hashlib

import numpy as np


def checksum(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()[:16]


ROUTER_CASES = {"a": (512, 64, 32, 4), "b": (96, 64, 16, 2), "c": (64, 64, 64, 8)}


def router_case(tag: str):
    """hidden [1,N,D] fp32 and router logits weight [E,D] fp32."""
    n, d, e, k = ROUTER_CASES[tag]
    rng = np.random.default_rng(1000 + ord(tag))
    weight = rng.normal(0, 0.2, (e, d)).astype(np.float32)
    hidden = rng.normal(0, 1, (1, n, d)).astype(np.float32)
    return dict(hidden=hidden, weight=weight, k=k)


MOE_CASES = {"a": (96, 64, 8, 2, 32), "b": (40, 64, 8, 4, 32)}


def moe_case(tag: str):
    """flat [N,D], router logits [N,E], expert stacks (moe.py:119-125 layout)."""
    n, d, e, k, f = MOE_CASES[tag]
    rng = np.random.default_rng(2000 + ord(tag))
    return dict(
        flat=rng.normal(0, 1, (n, d)).astype(np.float32),
        logits=rng.normal(0, 1, (n, e)).astype(np.float32),
        w_gate=rng.normal(0, 0.05, (e, f, d)).astype(np.float32),
        w_up=rng.normal(0, 0.05, (e, f, d)).astype(np.float32),
        w_down=rng.normal(0, 0.05, (e, d, f)).astype(np.float32),
        k=k,
    )


GDN_CASES = {"a": (2, 40, 64, 2, 64, 64), "b": (1, 130, 128, 2, 64, 64)}


def gdn_case(tag: str):
    """GatedDeltaNet weights (reference parameter names), input, state and resets."""
    b, t, d, h, kd, vd = GDN_CASES[tag]
    rng = np.random.default_rng(3000 + ord(tag))
    w = lambda *s: rng.normal(0, 0.1, s).astype(np.float32)
    p = dict(q_proj=w(h * kd, d), k_proj=w(h * kd, d), v_proj=w(h * vd, d), beta_proj=w(h, d),
             beta_bias=w(h), gate_proj=w(h * vd, d), out_proj=w(d, h * vd), conv=w(d, 1, 4),
             decay_logit=rng.uniform(0.5, 3.0, h).astype(np.float32))
    hidden = rng.normal(0, 1, (b, t, d)).astype(np.float32)
    state = rng.normal(0, 0.3, (b, h, kd, vd)).astype(np.float32)
    reset = np.zeros((b, t), dtype=bool)
    reset[0, t // 3] = True
    steps = rng.normal(0, 1, (b, 3, d)).astype(np.float32)  # decode tokens after the prefix
    return dict(p=p, hidden=hidden, state=state, reset=reset, steps=steps, heads=h, key_dim=kd,
                value_dim=vd)


CSA_CASES = {"a": (1, 100, 64, 4, 16, 32), "b": (2, 70, 96, 3, 32, 128)}


def csa_case(tag: str):
    """CSA weights (reference parameter names), input and decode tokens."""
    b, t, d, h, dh, w = CSA_CASES[tag]
    rng = np.random.default_rng(4000 + ord(tag))
    m = lambda *s: rng.normal(0, 0.15, s).astype(np.float32)
    p = dict(query=m(h * dh, d), key=m(h * dh, d), value=m(d, d), local_out=m(d, d),
             remote_out=m(d, d), out=m(d, d))
    hidden = rng.normal(0, 1, (b, t, d)).astype(np.float32)
    steps = rng.normal(0, 1, (b, 3, d)).astype(np.float32)
    return dict(p=p, hidden=hidden, steps=steps, heads=h, head_dim=dh, window=w)


BAND_CASES = {"a": (2, 90, 3, 16, 16, 24, 3), "b": (1, 64, 2, 32, 32, 64, 1)}


def band_case(tag: str):
    """q,k [B,T,H,D], v [B,T,Hv,Dv] for the per-head banded SDPA."""
    b, t, h, d, dv, w, hv = BAND_CASES[tag]
    rng = np.random.default_rng(5000 + ord(tag))
    return dict(q=rng.normal(size=(b, t, h, d)).astype(np.float32),
                k=rng.normal(size=(b, t, h, d)).astype(np.float32),
                v=rng.normal(size=(b, t, hv, dv)).astype(np.float32), window=w)


SAMPLE_CASES = {
    "greedy": dict(temp=0.0, top_k=50, top_p=0.9, rep=1.1),
    "topk": dict(temp=0.7, top_k=50, top_p=1.0, rep=1.0),
    "topk_topp": dict(temp=0.7, top_k=50, top_p=0.9, rep=1.1),
    "topp_only": dict(temp=1.3, top_k=0, top_p=0.8, rep=1.2),
    "temp_only": dict(temp=0.9, top_k=0, top_p=1.0, rep=1.0),
    "topk_big": dict(temp=1.0, top_k=700, top_p=0.95, rep=1.05),
}


def sample_case(tag: str):
    """logits [4, 1000] (a few sharp rows), generated ids per row, uniforms."""
    rng = np.random.default_rng(6000 + sum(map(ord, tag)))
    logits = rng.normal(0, 2.0, (4, 1000)).astype(np.float32)
    logits[1] *= 4.0
    generated = [rng.integers(0, 1000, size=n).tolist() for n in (0, 5, 40, 200)]
    # the rows with many repeats get penalised ids among their top logits
    generated[2] += np.argsort(-logits[2])[:3].tolist()
    uniforms = rng.uniform(0, 1, 4).astype(np.float32)
    return dict(logits=logits, generated=generated, uniforms=uniforms, **SAMPLE_CASES[tag])


def mini_config():
    """A small looped hybrid model inside every kernel's supported shapes."""
    from hybrid_llm_b200.config import HybridConfig
    return HybridConfig(vocab_size=1000, d_model=256, recurrent_layout=("csa_moe", "gdn_moe"),
                        num_loops=2, gdn_heads=2, gdn_key_dim=64, gdn_value_dim=64, csa_heads=4,
                        csa_head_dim=64, csa_window=32, moe_experts=8, moe_top_k=2, moe_hidden=128,
                        name="mini")


def mhc_config():
    """The mini model with four hyper-connection streams (mhc.py defaults: 10
    Sinkhorn iterations, shared across loops, streams kept across loops)."""
    import dataclasses
    return dataclasses.replace(mini_config(), mhc_streams=4, mhc_iterations=10, name="mini-mhc")


def router_ctx_config():
    """The mini model with the context-aware router: 64-wide latents averaged
    over the last 8 tokens (the 50-token prompt fills the window)."""
    import dataclasses
    return dataclasses.replace(mini_config(), router_context=True, router_latent_dim=64,
                               router_local_context=8, name="mini-router-ctx")


def csa_remote_config():
    """The mini model with the CSA remote branch on: 4-token block summaries,
    top-3 per query and head (the 50-token prompt gives 12 summaries)."""
    import dataclasses
    return dataclasses.replace(mini_config(), csa_compression=4, csa_top_k=3,
                               name="mini-csa-remote")


def shared_experts_config():
    """The mini model with two shared experts next to the routed ones."""
    import dataclasses
    return dataclasses.replace(mini_config(), moe_shared=2, name="mini-shared")


def loop_memory_config():
    """The mini model with the loop memory between loops, three loops so that
    the last loop attends over two endpoints (LoopMemoryHook defaults:
    latent 128, 4 heads x 32)."""
    import dataclasses
    return dataclasses.replace(mini_config(), num_loops=3, loop_memory=True, name="mini-loop-mem")


def combined_config():
    """mHC (4 streams), the router's local context, the CSA remote branch and
    shared experts together on the mini model (their interaction)."""
    import dataclasses
    return dataclasses.replace(mini_config(), mhc_streams=4, mhc_iterations=10,
                               router_context=True, router_latent_dim=64, router_local_context=8,
                               csa_compression=4, csa_top_k=3, moe_shared=2, name="mini-combined")


def llmy_config():
    """A small looped hybrid model for the .llmy format fixture."""
    from hybrid_llm_b200.config import HybridConfig
    return HybridConfig(vocab_size=256, d_model=128, recurrent_layout=("csa_moe", "gdn_moe"),
                        num_loops=2, gdn_heads=2, gdn_key_dim=64, gdn_value_dim=64, csa_heads=2,
                        csa_head_dim=64, csa_window=16, moe_experts=4, moe_top_k=2, moe_hidden=128,
                        name="llmy-tiny")


def mini_prompt():
    rng = np.random.default_rng(7000)
    return rng.integers(0, 1000, size=(2, 50)).astype(np.int64)


def block_hidden():
    """Single-block workload input: hidden [1, 256, 512] ~ N(0, 1)."""
    return np.random.default_rng(1).normal(0, 1, (1, 256, 512)).astype(np.float32)


def v6_mapping(cfg) -> dict:
    """Reference V6Config fields for a HybridConfig (mHC, the router's local
    context path, the CSA remote branch, shared experts and the loop memory as
    configured; adaptive halting switched off)."""
    return dict(
        vocab_size=cfg.vocab_size, d_model=cfg.d_model, physical_blocks=cfg.n_blocks,
        stem_blocks=0, recurrent_blocks=cfg.n_blocks, tail_blocks=0, num_loops=cfg.num_loops,
        recurrent_layout=list(cfg.recurrent_layout),
        mhc=(dict(enabled=True, streams=cfg.mhc_streams, sinkhorn_iterations=cfg.mhc_iterations,
                  shared_across_loops=True, preserve_streams_across_loop_boundary=True)
             if cfg.mhc_streams else dict(enabled=False, streams=1)),
        gdn=dict(qk_heads=cfg.gdn_heads, value_heads=cfg.gdn_heads, qk_head_dim=cfg.gdn_key_dim,
                 value_head_dim=cfg.gdn_value_dim, conv_kernel=cfg.conv_kernel),
        moe=dict(routed_experts=cfg.moe_experts, shared_experts=cfg.moe_shared,
                 routed_top_k=cfg.moe_top_k, expert_hidden=cfg.moe_hidden),
        router=dict(context_aware=cfg.router_context, local_context=cfg.router_local_context),
        mla=dict(latent_dim=cfg.router_latent_dim),
        csa=dict(temporal_compression=cfg.csa_compression or 10 ** 9, local_window=cfg.csa_window,
                 index_heads=cfg.csa_heads, index_head_dim=cfg.csa_head_dim,
                 index_top_k=cfg.csa_top_k if cfg.csa_compression else 4),
        loop_attnres=dict(enabled=cfg.loop_memory, latent_dim=cfg.loop_memory_latent,
                          heads=cfg.loop_memory_heads, head_dim=cfg.loop_memory_head_dim),
        adaptive_loops=dict(enabled=False),
    )
