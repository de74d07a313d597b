"""Model configuration of the looped hybrid stack served by this package.

Mirrors the parts of the reference V6Config (model/config.py:107-191) that the
B200 path implements: a recurrent core of ``gdn_moe`` / ``csa_moe`` blocks run
``num_loops`` times, with either one plain residual stream (mHC disabled,
``mhc_streams == 0``) or multi-stream hyper-connections (``mhc_streams`` = 1, 2
or 4 live streams, input-dependent maps, shared across loops, streams carried
across loop boundaries), a top-k softmax router with or without its local
context path (``router_context``: the causal box-filtered MLA latents of the
last ``router_local_context`` tokens; no HCA global latents), routed and
shared experts (``moe_shared``), CSA with or without its remote compressed
branch (``csa_compression``), the loop memory between loops (``loop_memory``),
no stem/tail blocks and no adaptive halting.  ``from_v6`` converts a
reference config (dataclass or mapping) and rejects anything outside that
subset instead of silently changing the model.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any


# A CSA temporal_compression at least this large (16M tokens; the reference's
# own "off" setting is 10**9) completes no block in any sequence the engine
# holds, so its remote branch contributes exactly zero.
CSA_COMPRESSION_OFF = 1 << 24


@dataclass(frozen=True)
class HybridConfig:
    vocab_size: int
    d_model: int
    recurrent_layout: tuple[str, ...]
    num_loops: int
    gdn_heads: int
    gdn_key_dim: int
    gdn_value_dim: int
    csa_heads: int
    csa_head_dim: int
    csa_window: int
    moe_experts: int
    moe_top_k: int
    moe_hidden: int
    conv_kernel: int = 4
    rms_eps: float = 1e-6
    mhc_streams: int = 0          # 0: plain residual; S > 0: S-stream hyper-connections
    mhc_iterations: int = 10      # Sinkhorn iterations of the residual map
    router_context: bool = False  # ContextAwareRouter local-context path (context_router.py)
    router_latent_dim: int = 256  # mla.latent_dim
    router_local_context: int = 128  # router.local_context (box-filter window)
    # CSA remote compressed branch: block ratio (0 = off: temporal_compression
    # beyond any sequence) and summaries attended per query and head
    csa_compression: int = 0
    csa_top_k: int = 32
    moe_shared: int = 0  # shared experts (moe.py:185-198): sum of their SwiGLU / sqrt(n)
    # loop memory (loop_memory.py LoopMemoryHook, config loop_attnres): before
    # every loop after the first, each token attends over LayerNorm'd latent
    # summaries of its own streams at the end of the earlier loops
    loop_memory: bool = False
    loop_memory_latent: int = 128
    loop_memory_heads: int = 4
    loop_memory_head_dim: int = 32
    name: str = field(default="custom", compare=False)

    def __post_init__(self) -> None:
        for kind in self.recurrent_layout:
            if kind not in ("gdn_moe", "csa_moe"):
                raise ValueError(f"unsupported block kind {kind!r} (gdn_moe or csa_moe)")
        if self.num_loops < 1:
            raise ValueError("num_loops must be positive")
        if self.moe_top_k > self.moe_experts:
            raise ValueError("moe_top_k cannot exceed moe_experts")
        if self.conv_kernel != 4:
            raise ValueError("the GDN conv gate kernel implements kernel size 4")
        if self.mhc_streams not in (0, 1, 2, 4):
            raise ValueError("hyper-connections are implemented for 1, 2 or 4 streams")
        if self.mhc_iterations < 0:
            raise ValueError("mhc_iterations must be >= 0")
        if self.moe_shared < 0:
            raise ValueError("moe_shared must be >= 0")
        if self.csa_compression < 0 or self.csa_top_k < 1:
            raise ValueError("csa_compression must be >= 0 and csa_top_k >= 1")
        if self.router_context and (self.router_local_context < 1 or self.router_latent_dim < 1
                                    or self.router_latent_dim > 1024):
            raise ValueError("router context needs local_context >= 1 and 1 <= latent_dim <= 1024")
        if self.loop_memory and (self.loop_memory_latent < 1 or self.loop_memory_heads < 1
                                 or self.loop_memory_head_dim < 1 or self.num_loops > 16):
            raise ValueError("loop memory needs positive latent / head sizes and at most 16 loops")

    @property
    def streams(self) -> int:
        """Residual streams carried per token (1 without hyper-connections)."""
        return max(1, self.mhc_streams)

    @property
    def n_blocks(self) -> int:
        return len(self.recurrent_layout)

    def block_kind(self, j: int) -> str:
        return self.recurrent_layout[j].split("_")[0]

    @classmethod
    def from_v6(cls, cfg: Any) -> "HybridConfig":
        """Convert a reference V6Config (or the mapping its checkpoints embed)."""
        get = (lambda o, k: o[k]) if isinstance(cfg, dict) else getattr
        sub = lambda name: get(cfg, name)
        sget = lambda o, k: o[k] if isinstance(o, dict) else getattr(o, k)
        mhc = sub("mhc")
        mget = lambda k, default: (mhc.get(k, default) if isinstance(mhc, dict)
                                   else getattr(mhc, k, default))
        mhc_streams, mhc_iters = 0, 10
        if mget("enabled", True):
            mhc_streams, mhc_iters = int(mget("streams", 4)), int(mget("sinkhorn_iterations", 10))
            if not mget("shared_across_loops", True):
                raise ValueError("per-loop hyper-connection weights are not implemented")
            if not mget("preserve_streams_across_loop_boundary", True):
                raise ValueError("restarting the streams at each loop is not implemented")
        elif int(mget("streams", 1)) != 1:
            raise ValueError("mHC disabled with several streams is not implemented")
        router = sub("router")
        rget = lambda k, default: (router.get(k, default) if isinstance(router, dict)
                                   else getattr(router, k, default))
        router_context = bool(rget("context_aware", True))
        local_context = int(rget("local_context", 128))
        mla = sub("mla") if (isinstance(cfg, dict) and "mla" in cfg) or hasattr(cfg, "mla") else {}
        latent_dim = int(mla.get("latent_dim", 256) if isinstance(mla, dict)
                         else getattr(mla, "latent_dim", 256))
        gdn = sub("gdn")
        gget = lambda k, default: (gdn.get(k, default) if isinstance(gdn, dict)
                                   else getattr(gdn, k, default))
        if str(gget("sensitive_state_dtype", "float32")).lower() not in ("float32", "fp32"):
            # model/model.py:93 keeps the delta-rule state in fp16 then; this
            # build keeps it in fp32 only
            raise ValueError("the GDN state is kept in float32 only (gdn.sensitive_state_dtype)")
        if int(gget("value_heads", gget("qk_heads", 0))) != int(gget("qk_heads", 0)):
            raise ValueError("GDN needs equal q/k and value head counts (gated_deltanet.py:93)")
        if sub("stem_blocks") or sub("tail_blocks"):
            raise ValueError("stem/tail dense blocks are not implemented")
        if sget(sub("adaptive_loops"), "enabled"):
            raise ValueError("adaptive halting is not implemented")
        lm = sub("loop_attnres")
        lmget = lambda k, default: (lm.get(k, default) if isinstance(lm, dict)
                                    else getattr(lm, k, default))
        csa = sub("csa")
        ratio = int(sget(csa, "temporal_compression"))
        csa_compression = 0 if ratio >= CSA_COMPRESSION_OFF else ratio
        csa_top_k = int(sget(csa, "index_top_k")) if csa_compression else 32
        return cls(
            vocab_size=sub("vocab_size"), d_model=sub("d_model"),
            recurrent_layout=tuple(sub("recurrent_layout")), num_loops=sub("num_loops"),
            gdn_heads=sget(sub("gdn"), "qk_heads"), gdn_key_dim=sget(sub("gdn"), "qk_head_dim"),
            gdn_value_dim=sget(sub("gdn"), "value_head_dim"),
            csa_heads=sget(csa, "index_heads"), csa_head_dim=sget(csa, "index_head_dim"),
            csa_window=sget(csa, "local_window"),
            moe_experts=sget(sub("moe"), "routed_experts"), moe_top_k=sget(sub("moe"), "routed_top_k"),
            moe_hidden=sget(sub("moe"), "expert_hidden"),
            conv_kernel=sget(sub("gdn"), "conv_kernel"),
            mhc_streams=mhc_streams, mhc_iterations=mhc_iters,
            router_context=router_context, router_latent_dim=latent_dim,
            router_local_context=local_context,
            csa_compression=csa_compression, csa_top_k=csa_top_k,
            moe_shared=int(sget(sub("moe"), "shared_experts")),
            loop_memory=bool(lmget("enabled", False)),
            loop_memory_latent=int(lmget("latent_dim", 128)),
            loop_memory_heads=int(lmget("heads", 4)),
            loop_memory_head_dim=int(lmget("head_dim", 32)),
        )


def single_block_config() -> HybridConfig:
    """The single looped hybrid block workload (csa_moe + gdn_moe, d=512, 2 loops)."""
    return HybridConfig(vocab_size=32000, d_model=512, recurrent_layout=("csa_moe", "gdn_moe"),
                        num_loops=2, gdn_heads=8, gdn_key_dim=64, gdn_value_dim=64, csa_heads=8,
                        csa_head_dim=64, csa_window=128, moe_experts=8, moe_top_k=2,
                        moe_hidden=1024, name="single-block")


def small_llmy_config() -> HybridConfig:
    """Full small LLMY model: vocab 32000, d 768, 12 alternating blocks, 16 experts top-2."""
    return HybridConfig(vocab_size=32000, d_model=768, recurrent_layout=("csa_moe", "gdn_moe") * 6,
                        num_loops=2, gdn_heads=12, gdn_key_dim=64, gdn_value_dim=64, csa_heads=12,
                        csa_head_dim=64, csa_window=512, moe_experts=16, moe_top_k=2,
                        moe_hidden=1024, name="small-llmy")


def large_ep_config() -> HybridConfig:
    """Expert-parallel large model: d 2048, 24 blocks, 64 experts top-8, 3 loops, vocab 64000."""
    return HybridConfig(vocab_size=64000, d_model=2048, recurrent_layout=("csa_moe", "gdn_moe") * 12,
                        num_loops=3, gdn_heads=16, gdn_key_dim=128, gdn_value_dim=128, csa_heads=16,
                        csa_head_dim=128, csa_window=2048, moe_experts=64, moe_top_k=8,
                        moe_hidden=1024, name="large-ep")
