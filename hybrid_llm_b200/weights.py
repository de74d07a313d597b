"""Weights of the looped hybrid stack in the kernels' device layout.

Parameter names follow the reference state dict (model/model.py:383-423 and
the layer modules), so a reference checkpoint's tensors load directly:
  embed_tokens.weight [V,D]; stream_seed [S,D]; mhc_collapse.weight [D,S*D];
  final_norm.weight [D]; recurrent_core.{j}.mixer_norm.weight / ffn_norm.weight;
  mHC  recurrent_core.{j}.mhc.{stream_scale [S,D], stream_norm.{weight,bias} [D],
       mapping_norm.weight [S*D], theta.weight [2S+S*S, S*D], pre_bias [S],
       post_bias [S], residual_bias [S,S], alpha_pre, alpha_post, alpha_residual,
       gating_logit, read_logits, write_logits}        (mhc.py:62-88; S streams)
  router context  recurrent_core.{j}.moe.router.{latent_memory.down.weight [L,D],
       latent_memory.norm.{weight,bias} [L], local_context_out.weight [D,L],
       context_out.weight [D,D], route_gate}         (context_router.py:14-27)
  GDN  recurrent_core.{j}.mixer.{q,k,v,gate,out}_proj.weight, beta_proj.{weight,bias},
       conv.weight [D,1,4], decay_logit [H]          (gated_deltanet.py:105-113)
  CSA  recurrent_core.{j}.mixer.{query,key,value,local_out,out}.weight  (csa.py:23-28)
  MoE  recurrent_core.{j}.moe.router.norm.weight, moe.router.logits.weight [E,D],
       moe.experts.{e}.{gate,up,down}_proj.weight   (moe.py:104-110, expert.py)
Device layout: the GDN q/k/v/gate/beta projections are fused into one
[P, D] matrix (P padded to a multiple of 8 for 16-byte rows), the CSA
query/key/value into one [2*H*Dh + D, D] matrix, and the experts into the
interleaved gate/up stack w13 [E, 2F, D] plus w2 [E, D, F] (bf16).  The CSA
output path out(local_out(x)) (csa.py:132) is also kept as the single
product matrix w_o = W_out W_local_out (formed in fp32) for decode, which
halves its weight traffic per token.

``synthetic_state_dict`` draws the random-init weights of the benchmark
workloads: every tensor with two or more dimensions ~ N(0, 0.02), norm
weights 1, beta bias 0, decay_logit 2 (the reference's own 1-D inits).  The
hyper-connection parameters get values that exercise every term of the maps
instead of the reference's near-identity init: theta ~ N(0, 0.02); scales,
norm weights ~ 1 + N(0, 0.1); biases ~ N(0, 0.1) around the reference's
(logit(1/S) for pre, 4·I for the residual map, with N(0, 0.5)); alphas 0.3;
gating factor 0.3.  Each
tensor from its own generator seeded by (seed, name) so that any subset can
be regenerated identically on any machine (CPU generation) or quickly on the
GPU (CUDA generation).
"""
from __future__ import annotations

import zlib
from dataclasses import dataclass
from typing import Callable, Mapping

import torch

from . import kernels
from .config import HybridConfig


def parameter_shapes(cfg: HybridConfig) -> dict[str, tuple[int, ...]]:
    """Every reference parameter name the B200 path reads, with its shape."""
    d, e, f = cfg.d_model, cfg.moe_experts, cfg.moe_hidden
    ns = cfg.streams
    shapes: dict[str, tuple[int, ...]] = {
        "embed_tokens.weight": (cfg.vocab_size, d), "stream_seed": (ns, d),
        "mhc_collapse.weight": (d, ns * d), "final_norm.weight": (d,),
    }
    for j in range(cfg.n_blocks):
        p = f"recurrent_core.{j}."
        shapes[p + "mixer_norm.weight"] = (d,)
        shapes[p + "ffn_norm.weight"] = (d,)
        if cfg.mhc_streams:
            q = p + "mhc."
            shapes.update({
                q + "read_logits": (ns, ns), q + "write_logits": (ns, ns),
                q + "stream_scale": (ns, d), q + "stream_norm.weight": (d,),
                q + "stream_norm.bias": (d,), q + "mapping_norm.weight": (ns * d,),
                q + "theta.weight": (2 * ns + ns * ns, ns * d), q + "pre_bias": (ns,),
                q + "post_bias": (ns,), q + "residual_bias": (ns, ns), q + "alpha_pre": (),
                q + "alpha_post": (), q + "alpha_residual": (), q + "gating_logit": (),
            })
        if cfg.block_kind(j) == "gdn":
            h, kd, vd = cfg.gdn_heads, cfg.gdn_key_dim, cfg.gdn_value_dim
            shapes.update({
                p + "mixer.q_proj.weight": (h * kd, d), p + "mixer.k_proj.weight": (h * kd, d),
                p + "mixer.v_proj.weight": (h * vd, d), p + "mixer.beta_proj.weight": (h, d),
                p + "mixer.beta_proj.bias": (h,), p + "mixer.gate_proj.weight": (h * vd, d),
                p + "mixer.out_proj.weight": (d, h * vd), p + "mixer.conv.weight": (d, 1, cfg.conv_kernel),
                p + "mixer.decay_logit": (h,),
            })
        else:
            w = cfg.csa_heads * cfg.csa_head_dim
            shapes.update({
                p + "mixer.query.weight": (w, d), p + "mixer.key.weight": (w, d),
                p + "mixer.value.weight": (d, d), p + "mixer.local_out.weight": (d, d),
                p + "mixer.out.weight": (d, d),
            })
            if cfg.csa_compression:
                shapes.update({
                    p + "mixer.remote_out.weight": (d, d),
                    p + "mixer.compressor.key.weight": (w, d),
                    p + "mixer.compressor.value.weight": (d, d),
                })
        shapes[p + "moe.router.norm.weight"] = (d,)
        shapes[p + "moe.router.logits.weight"] = (e, d)
        if cfg.router_context:
            q, lat = p + "moe.router.", cfg.router_latent_dim
            shapes.update({
                q + "latent_memory.down.weight": (lat, d), q + "latent_memory.norm.weight": (lat,),
                q + "latent_memory.norm.bias": (lat,), q + "local_context_out.weight": (d, lat),
                q + "context_out.weight": (d, d), q + "route_gate": (),
            })
        for x in range(e):
            q = f"{p}moe.experts.{x}."
            shapes[q + "gate_proj.weight"] = (f, d)
            shapes[q + "up_proj.weight"] = (f, d)
            shapes[q + "down_proj.weight"] = (d, f)
        for x in range(cfg.moe_shared):
            q = f"{p}moe.shared.{x}."
            shapes[q + "gate_proj.weight"] = (f, d)
            shapes[q + "up_proj.weight"] = (f, d)
            shapes[q + "down_proj.weight"] = (d, f)
    if cfg.loop_memory:
        q, lat = "loop_memory.", cfg.loop_memory_latent
        w = cfg.loop_memory_heads * cfg.loop_memory_head_dim
        shapes.update({
            q + "compressor.down.weight": (lat, d), q + "compressor.up.weight": (d, lat),
            q + "compressor.norm.weight": (lat,), q + "compressor.norm.bias": (lat,),
            q + "query_norm.weight": (d,), q + "query_norm.bias": (d,),
            q + "attention.q.weight": (w, d), q + "attention.k.weight": (w, lat),
            q + "attention.v.weight": (w, lat), q + "attention.o.weight": (d, w),
            q + "gating_logit": (),
        })
    return shapes


class LazyStateDict(Mapping):
    """Read-only mapping name -> tensor that materialises tensors on access."""

    def __init__(self, shapes: dict[str, tuple[int, ...]], make: Callable[[str, tuple], torch.Tensor]):
        self._shapes = shapes
        self._make = make

    def __getitem__(self, name: str) -> torch.Tensor:
        return self._make(name, self._shapes[name])

    def __iter__(self):
        return iter(self._shapes)

    def __len__(self) -> int:
        return len(self._shapes)


def synthetic_state_dict(cfg: HybridConfig, seed: int = 0, device: str | torch.device = "cpu",
                         std: float = 0.02) -> LazyStateDict:
    device = torch.device(device)

    def noise(name: str, shape: tuple, scale: float) -> torch.Tensor:
        gen = torch.Generator(device=device)
        gen.manual_seed((seed * 1_000_003 + zlib.crc32(name.encode())) % (2 ** 62))
        return torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * scale

    def make_mhc(name: str, shape: tuple) -> torch.Tensor:
        leaf = name.rsplit("mhc.", 1)[1]
        ns = cfg.streams
        if leaf in ("read_logits", "write_logits"):
            return torch.eye(ns, device=device) * 4.0
        if leaf == "theta.weight":
            return noise(name, shape, std)
        if leaf in ("stream_scale", "stream_norm.weight", "mapping_norm.weight"):
            return 1.0 + noise(name, shape, 0.1)
        if leaf == "stream_norm.bias" or leaf == "post_bias":
            return noise(name, shape, 0.1)
        if leaf == "pre_bias":
            return torch.logit(torch.tensor(1.0 / ns)) + noise(name, shape, 0.1)
        if leaf == "residual_bias":
            return torch.eye(ns, device=device) * 4.0 + noise(name, shape, 0.5)
        if leaf.startswith("alpha_"):
            return torch.tensor(0.3, device=device)
        if leaf == "gating_logit":
            return torch.logit(torch.tensor(0.3)).to(device)
        raise KeyError(name)

    def make_loop_memory(name: str, shape: tuple) -> torch.Tensor:
        if name.endswith("gating_logit"):
            return torch.zeros(shape, device=device)  # gate sigmoid(0) = 0.5
        if name.endswith("norm.weight"):
            return 1.0 + noise(name, shape, 0.1)
        if name.endswith("norm.bias"):
            return noise(name, shape, 0.1)
        return noise(name, shape, 0.1)

    def make(name: str, shape: tuple) -> torch.Tensor:
        if ".mhc." in name:
            return make_mhc(name, shape)
        if name.startswith("loop_memory."):
            return make_loop_memory(name, shape)
        if len(shape) >= 2:
            gen = torch.Generator(device=device)
            gen.manual_seed((seed * 1_000_003 + zlib.crc32(name.encode())) % (2 ** 62))
            return torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std
        if name.endswith("beta_proj.bias") or name.endswith("latent_memory.norm.bias"):
            return torch.zeros(shape, device=device)
        if name.endswith("route_gate"):
            # sigmoid(0) = 0.5 (the reference's init, -4.595, gives 0.01) so that
            # the local context visibly moves the routing logits
            return torch.zeros(shape, device=device)
        if name.endswith("decay_logit"):
            return torch.full(shape, 2.0, device=device)
        return torch.ones(shape, device=device)  # norm weights

    return LazyStateDict(parameter_shapes(cfg), make)


@dataclass
class GdnBlock:
    w_in: torch.Tensor       # [P, D] bf16: q | k | v | gate | beta | zero pad
    beta_bias: torch.Tensor  # [H] fp32
    decay_logit: torch.Tensor  # [H] fp32
    w_out: torch.Tensor      # [D, H*V] bf16
    conv: torch.Tensor       # [D, 4] fp32


@dataclass
class CsaBlock:
    w_in: torch.Tensor       # [2*H*Dh + D, D] bf16: query | key | value
    local_out: torch.Tensor  # [D, D] bf16
    out: torch.Tensor        # [D, D] bf16
    # decode output projection (computed in fp32): out @ local_out [D, D], or
    # with the remote branch [out @ local_out | out @ remote_out] [D, 2D]
    w_o: torch.Tensor
    # remote branch (None without it): remote_out [D, D] and the compressor's
    # [key; value] [H*Dh + D, D] (compressed_attention.py:80-83), bf16
    remote_out: torch.Tensor | None = None
    w_comp: torch.Tensor | None = None


@dataclass
class MoeBlock:
    router_norm: torch.Tensor  # [D] fp32
    router: torch.Tensor       # [E, D] fp32
    w13: torch.Tensor          # [E+S, 2F, D] bf16 (interleaved gate/up; routed, then S shared)
    w2: torch.Tensor           # [E+S, D, F] bf16
    router_folded: torch.Tensor | None = None  # [E, D] fp32 = router * ffn_norm * router_norm
    # local-context path of the ContextAwareRouter (None without it)
    ctx_down: torch.Tensor | None = None   # [L, D] fp32 latent_memory.down
    ctx_ln_w: torch.Tensor | None = None   # [L] fp32 latent_memory.norm (LayerNorm)
    ctx_ln_b: torch.Tensor | None = None   # [L] fp32
    ctx_logits: torch.Tensor | None = None  # [E, L] fp32 = router @ context_out @ local_context_out
    ctx_gate: float = 0.0                  # sigmoid(route_gate)


@dataclass
class MhcBlock:
    """One block's hyper-connection (mhc.py:52-229) in the kernels' layout."""
    theta: torch.Tensor         # [2S+S*S, S*D] fp32: theta.weight * mapping_norm.weight (columns)
    stream_scale: torch.Tensor  # [S, D] fp32
    ln_w: torch.Tensor          # [D] fp32 stream_norm (LayerNorm) weight
    ln_b: torch.Tensor          # [D] fp32 stream_norm bias
    bias: torch.Tensor          # [2S+S*S] fp32: pre_bias | post_bias | residual_bias
    scalars: torch.Tensor       # [4] fp32: alpha_pre, alpha_post, alpha_residual, sigmoid(gating)
    static: bool = False        # theta is all zero: input-independent maps (mhc.py:114-118)


@dataclass
class LoopMemory:
    """The loop memory hook (loop_memory.py:11-66) in fp32: latent compressor
    (down, LayerNorm), query LayerNorm, latent attention and its gate."""
    down: torch.Tensor      # [L, D]
    lat_w: torch.Tensor     # [L] compressor LayerNorm
    lat_b: torch.Tensor     # [L]
    q_ln_w: torch.Tensor    # [D] query LayerNorm
    q_ln_b: torch.Tensor    # [D]
    wq: torch.Tensor        # [H*hd, D]
    wkv: torch.Tensor       # [2*H*hd, L]: k rows, then v rows
    wo: torch.Tensor        # [D, H*hd]
    gate: float             # sigmoid(gating_logit)


@dataclass
class Block:
    kind: str
    mixer_norm: torch.Tensor
    ffn_norm: torch.Tensor
    mixer: GdnBlock | CsaBlock
    moe: MoeBlock
    mhc: MhcBlock | None = None


def _experts(sd: Mapping[str, torch.Tensor], p: str, name: str, lo: int, hi: int,
             dev: torch.device, group: str = "experts") -> torch.Tensor:
    """Experts lo..hi-1 of one projection as [hi-lo, rows, cols] bf16: from the
    per-expert parameters (moe.<group>.<e>.<name>.weight) or from one stacked
    tensor (moe.<group>.<name>.weight, the .llmy converter's layout); group
    "experts" (routed) or "shared"."""
    stacked = sd.get(f"{p}moe.{group}.{name}.weight")
    if stacked is not None:
        return stacked[lo:hi].to(dev, torch.bfloat16)
    return torch.stack([sd[f"{p}moe.{group}.{x}.{name}.weight"].to(dev, torch.bfloat16)
                        for x in range(lo, hi)])


def _expert_stack(sd, p: str, name: str, lo: int, hi: int, n_shared: int,
                  dev: torch.device) -> torch.Tensor:
    """Routed experts lo..hi-1, then the n_shared shared experts, of one projection."""
    routed = _experts(sd, p, name, lo, hi, dev)
    if not n_shared:
        return routed
    return torch.cat([routed, _experts(sd, p, name, 0, n_shared, dev, group="shared")])


@dataclass
class ModelWeights:
    cfg: HybridConfig
    embed: torch.Tensor       # [V, D] bf16 (tied LM head)
    stream_seed: torch.Tensor  # [S*D] fp32 (S = cfg.streams)
    collapse: torch.Tensor    # [D, S*D] bf16
    final_norm: torch.Tensor  # [D] fp32
    blocks: list[Block]
    loop_memory: LoopMemory | None = None

    @classmethod
    def from_state_dict(cls, cfg: HybridConfig, sd: Mapping[str, torch.Tensor],
                        device: str | torch.device = "cuda",
                        expert_range: tuple[int, int] | None = None) -> "ModelWeights":
        """expert_range (lo, hi): keep only experts lo..hi-1 (one rank's shard
        under expert parallelism); the router keeps all experts."""
        dev = torch.device(device)
        lo, hi = (0, cfg.moe_experts) if expert_range is None else expert_range
        bf = lambda n: sd[n].to(device=dev, dtype=torch.bfloat16).contiguous()
        f32 = lambda n: sd[n].to(device=dev, dtype=torch.float32).contiguous()
        blocks = []
        for j in range(cfg.n_blocks):
            p = f"recurrent_core.{j}."
            if cfg.block_kind(j) == "gdn":
                parts = [sd[p + f"mixer.{n}.weight"].to(dev, torch.bfloat16)
                         for n in ("q_proj", "k_proj", "v_proj", "gate_proj", "beta_proj")]
                rows = sum(x.shape[0] for x in parts)
                pad = (-rows) % 8
                if pad:
                    parts.append(torch.zeros(pad, cfg.d_model, dtype=torch.bfloat16, device=dev))
                mixer = GdnBlock(
                    w_in=torch.cat(parts).contiguous(), beta_bias=f32(p + "mixer.beta_proj.bias"),
                    decay_logit=f32(p + "mixer.decay_logit"), w_out=bf(p + "mixer.out_proj.weight"),
                    conv=f32(p + "mixer.conv.weight").reshape(cfg.d_model, -1).contiguous())
            else:
                w_o = (f32(p + "mixer.out.weight") @ f32(p + "mixer.local_out.weight"))
                remote_out = w_comp = None
                if cfg.csa_compression:
                    w_o = torch.cat([w_o, f32(p + "mixer.out.weight")
                                     @ f32(p + "mixer.remote_out.weight")], 1)
                    remote_out = bf(p + "mixer.remote_out.weight")
                    w_comp = torch.cat([bf(p + "mixer.compressor.key.weight"),
                                        bf(p + "mixer.compressor.value.weight")]).contiguous()
                mixer = CsaBlock(
                    w_in=torch.cat([bf(p + "mixer.query.weight"), bf(p + "mixer.key.weight"),
                                    bf(p + "mixer.value.weight")]).contiguous(),
                    local_out=bf(p + "mixer.local_out.weight"), out=bf(p + "mixer.out.weight"),
                    w_o=w_o.to(torch.bfloat16).contiguous(), remote_out=remote_out,
                    w_comp=w_comp)
            ns = cfg.moe_shared
            gate = _expert_stack(sd, p, "gate_proj", lo, hi, ns, dev)
            up = _expert_stack(sd, p, "up_proj", lo, hi, ns, dev)
            w13 = kernels.pack_w13(gate, up)
            del gate, up
            w2 = _expert_stack(sd, p, "down_proj", lo, hi, ns, dev).contiguous()
            moe = MoeBlock(router_norm=f32(p + "moe.router.norm.weight"),
                           router=f32(p + "moe.router.logits.weight"), w13=w13, w2=w2)
            moe.router_folded = kernels.fold_router(moe.router, f32(p + "ffn_norm.weight"),
                                                    moe.router_norm)
            if cfg.router_context:
                q = p + "moe.router."
                moe.ctx_down = f32(q + "latent_memory.down.weight")
                moe.ctx_ln_w = f32(q + "latent_memory.norm.weight")
                moe.ctx_ln_b = f32(q + "latent_memory.norm.bias")
                # logits = router (local + g context_out(local_context_out(box)))
                #        = router local + g (router context_out local_context_out) box
                moe.ctx_logits = (moe.router @ f32(q + "context_out.weight")
                                  @ f32(q + "local_context_out.weight")).contiguous()
                moe.ctx_gate = float(torch.sigmoid(sd[q + "route_gate"].reshape(()).float()))
            mhc = None
            if cfg.mhc_streams:
                q = p + "mhc."
                sc = lambda n: float(sd[q + n].reshape(()).float())
                mhc = MhcBlock(
                    theta=(f32(q + "theta.weight") * f32(q + "mapping_norm.weight")[None, :]
                           ).contiguous(),
                    stream_scale=f32(q + "stream_scale"), ln_w=f32(q + "stream_norm.weight"),
                    ln_b=f32(q + "stream_norm.bias"),
                    bias=torch.cat([f32(q + "pre_bias").reshape(-1), f32(q + "post_bias").reshape(-1),
                                    f32(q + "residual_bias").reshape(-1)]).contiguous(),
                    scalars=torch.tensor([sc("alpha_pre"), sc("alpha_post"), sc("alpha_residual"),
                                          float(torch.sigmoid(torch.tensor(sc("gating_logit"))))],
                                         dtype=torch.float32, device=dev))
                mhc.static = not bool(torch.count_nonzero(mhc.theta))
            blocks.append(Block(cfg.block_kind(j), f32(p + "mixer_norm.weight"),
                                f32(p + "ffn_norm.weight"), mixer, moe, mhc))
        ns = cfg.streams
        seed_t = f32("stream_seed")
        collapse = bf("mhc_collapse.weight")
        if seed_t.numel() != ns * cfg.d_model or tuple(collapse.shape) != (cfg.d_model, ns * cfg.d_model):
            raise ValueError(f"stream_seed / mhc_collapse do not match {ns} residual stream(s)")
        loop_memory = None
        if cfg.loop_memory:
            q = "loop_memory."
            loop_memory = LoopMemory(
                down=f32(q + "compressor.down.weight"), lat_w=f32(q + "compressor.norm.weight"),
                lat_b=f32(q + "compressor.norm.bias"), q_ln_w=f32(q + "query_norm.weight"),
                q_ln_b=f32(q + "query_norm.bias"), wq=f32(q + "attention.q.weight"),
                wkv=torch.cat([f32(q + "attention.k.weight"), f32(q + "attention.v.weight")]
                              ).contiguous(),
                wo=f32(q + "attention.o.weight"),
                gate=float(torch.sigmoid(sd[q + "gating_logit"].reshape(()).float())))
        return cls(cfg=cfg, embed=bf("embed_tokens.weight"),
                   stream_seed=seed_t.reshape(-1).contiguous(), collapse=collapse,
                   final_norm=f32("final_norm.weight"), blocks=blocks, loop_memory=loop_memory)

    @classmethod
    def from_llmy(cls, path, device: str | torch.device = "cuda",
                  expert_range: tuple[int, int] | None = None) -> "ModelWeights":
        """Load a checkpoint in the reference engine's ``.llmy`` format
        (llmy_cuda/tools/convert_checkpoint.py): its embedded configuration
        through HybridConfig.from_v6, its (expert-stacked) tensors through
        from_state_dict."""
        from .llmy_format import read_llmy
        f = read_llmy(path)
        try:
            cfg = HybridConfig.from_v6(f.config)
            return cls.from_state_dict(cfg, f.tensors, device, expert_range=expert_range)
        finally:
            f.close()

    def nbytes(self) -> int:
        total = 0
        for t in self._tensors():
            total += t.numel() * t.element_size()
        return total

    def _tensors(self):
        yield from (self.embed, self.stream_seed, self.collapse, self.final_norm)
        if self.loop_memory is not None:
            yield from (t for t in vars(self.loop_memory).values() if isinstance(t, torch.Tensor))
        for b in self.blocks:
            yield from (b.mixer_norm, b.ffn_norm)
            yield from vars(b.mixer).values()
            yield from (t for t in vars(b.moe).values() if isinstance(t, torch.Tensor))
            if b.mhc is not None:
                yield from vars(b.mhc).values()
