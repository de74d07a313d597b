"""Looped hybrid LLMY stack on the llmyb kernels: prefill forward and decode step.

Host-side mirror of LoopedHybridMoEForCausalLM.forward / decode_step
(model/model.py:530-707, :787-915) and PhysicalBlock.forward / forward_step
(:162-376) for the configuration subset in ``config.HybridConfig``:

    streams = embed(ids) + stream_seed                        (fp32 residual)
    for loop in range(num_loops):            state namespace "loop{i}.core.{j}"
        for block j:
            x = RMSNorm_mixer(streams)                           (bf16)
            streams += GDN(x)  |  CSA_local(x)
            m = RMSNorm_ffn(streams)
            streams += MoE(m)         router: top-k(softmax) over W_r RMSNorm(m)
    logits = embed^T RMSNorm_final(collapse(streams))        (tied LM head)

Every hot operation is an llmyb kernel (router + dispatch plan, grouped
SwiGLU experts, GDN scan/step + conv gate, banded/CSA attention, fused
residual-add RMSNorm, embedding, sampling); the dense projections are plain
cuBLAS GEMMs through torch.  There is no CPU path: every tensor lives on the
GPU and the kernels raise if the native library is missing.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import kernels
from .config import HybridConfig
from .state import RecurrentState, state_key
from .weights import Block, CsaBlock, GdnBlock, ModelWeights


@dataclass
class HybridOutput:
    """Subset of LoopedHybridOutput (model/model.py:67-73) the inference path fills."""

    logits: torch.Tensor
    state: RecurrentState


class LoopedHybridModel:
    """ep: an ExpertParallel group when the weights hold one rank's expert
    shard (ModelWeights.from_state_dict(..., expert_range=ep.expert_range));
    every rank of the group then runs the same calls on its own sequences."""

    def __init__(self, weights: ModelWeights, ep=None):
        if weights.cfg.moe_shared and ep is not None:
            raise NotImplementedError(
                "shared experts (moe.shared_experts) are served on one device only, not under "
                "expert parallelism")
        self.w = weights
        self.cfg: HybridConfig = weights.cfg
        self.device = weights.embed.device
        self.ep = ep
        # expert kernels of prefill and decode: "auto", "grouped" (tcgen05 GEMMs)
        # or "decode" (weight streaming); a fixed choice makes a single-device
        # and an expert-parallel run comparable bit for bit
        self.expert_path = "auto"
        # small-batch decode on the fused kernels (decode_norm_gemv /
        # decode_out_router) when the shapes allow; False forces the unfused path
        self.decode_fused = True
        # batch-1 decode as one persistent launch (persistent.py) when the model
        # is in its served subset; False keeps the per-sub-layer kernels
        self.decode_persistent = True
        self._counter = torch.zeros(1, dtype=torch.int32, device=self.device)
        # diagnostics: when a list, every MoE call appends its routed top-k
        # indices [N, k] (device tensors, in call order; inside a CUDA graph
        # capture these are the graph's own buffers, rewritten by each replay)
        self.route_log: list | None = None
        shard = weights.blocks[0].moe.w13.shape[0] if weights.blocks else None
        if ep is not None and shard != ep.experts_per_rank:
            raise ValueError("expert-parallel model needs the weights of this rank's experts only")

    # ------------------------------------------------------------- helpers
    def _gdn_views(self, proj: torch.Tensor, lead: tuple[int, ...]):
        c = self.cfg
        h, kd, vd = c.gdn_heads, c.gdn_key_dim, c.gdn_value_dim
        hk, hv = h * kd, h * vd
        q = proj[..., :hk].unflatten(-1, (h, kd))
        k = proj[..., hk:2 * hk].unflatten(-1, (h, kd))
        v = proj[..., 2 * hk:2 * hk + hv].unflatten(-1, (h, vd))
        gate = proj[..., 2 * hk + hv:2 * hk + 2 * hv].unflatten(-1, (h, vd))
        beta = proj[..., 2 * hk + 2 * hv:2 * hk + 2 * hv + h]
        return q, k, v, gate, beta

    def _router_logits(self, blk: Block, m_f32: torch.Tensor, state: RecurrentState, key: str,
                       bsz: int, t: int, step: bool, normed: bool = False) -> torch.Tensor:
        """ContextAwareRouter logits (context_router.py:59-74 prefill, :89-133
        decode step): local = RMSNorm(hidden); logits = W local, plus the local
        context term when the router has it (the window's latents kept in
        state.router_latents for the following decode steps).  normed: m_f32
        already holds local (add_rmsnorm_router formed it with the FFN norm)."""
        c = self.cfg
        if normed:
            r_in = m_f32
        else:
            r_in = torch.empty_like(m_f32)
            kernels.add_rmsnorm(m_f32, None, blk.moe.router_norm, c.rms_eps, out_f32=r_in)
        if not c.router_context:
            return torch.mm(r_in, blk.moe.router.t())
        return kernels.router_context_logits(
            r_in, blk.moe, c.router_local_context, batch=bsz, seq=t,
            ring=state.router_latents[key], positions=state.positions if step else None)

    def _router_in_fused(self) -> bool:
        """Prompt MoE sub-layers whose router input is formed together with the
        FFN norm (add_rmsnorm_router): where the one-kernel router
        (route_norm) does not take the shape."""
        c = self.cfg
        return ((c.router_context or not kernels.route_norm_supported(c.d_model, c.moe_experts))
                and kernels.add_rmsnorm_router_supported(c.d_model))

    def _moe(self, blk: Block, m_bf: torch.Tensor, m_f32: torch.Tensor, state: RecurrentState,
             key: str, bsz: int, t: int, normed: bool = False):
        """SparseMoE.forward (moe.py:172-204): the expert rows and the plan whose
        per-token sum is the combine (added to the residual stream by the next
        add_rmsnorm_routed).  normed: m_f32 is the router's input already."""
        c = self.cfg
        tile_m = kernels.grouped_tile_m(bsz * t * c.moe_top_k, c.moe_experts + c.moe_shared)
        if (not normed and not c.router_context
                and kernels.route_norm_supported(c.d_model, c.moe_experts)):
            plan = kernels.route_norm(m_f32, blk.moe.router_norm, blk.moe.router, c.moe_top_k,
                                      c.rms_eps, tile_m=tile_m)
        else:
            logits = self._router_logits(blk, m_f32, state, key, bsz, t, step=False,
                                         normed=normed)
            plan = kernels.route(logits, c.moe_top_k, tile_m=tile_m)
        return self._experts(blk, m_bf, plan)

    def _add_pending(self, streams, pending, weight, **out) -> None:
        """streams += pending (a bf16 delta, or routed expert rows + plan, whose
        per-token sum is the MoE combine), then RMSNorm into `out`."""
        if isinstance(pending, tuple):
            kernels.add_rmsnorm_routed(streams, pending[0], pending[1], weight, self.cfg.rms_eps,
                                       **out)
        else:
            kernels.add_rmsnorm(streams, pending, weight, self.cfg.rms_eps, **out)

    # --------------------------------------------------------- loop memory
    def _lm_buffer(self, n: int, loops: int) -> torch.Tensor | None:
        """k|v projections of the loop endpoints [loops-1, N, 2*H*hd] fp32."""
        c = self.cfg
        if not c.loop_memory or loops < 2:
            return None
        w = 2 * c.loop_memory_heads * c.loop_memory_head_dim
        return torch.empty(loops - 1, n, w, dtype=torch.float32, device=self.device)

    def _lm_record(self, streams: torch.Tensor, kv: torch.Tensor, i: int) -> None:
        """LoopMemoryHook.record / encode (loop_memory.py:36-38, :54-66) after
        loop i: endpoint = LayerNorm(down(mean over streams)), kept as its k|v
        projections for the later loops' attention."""
        c, lm = self.cfg, self.w.loop_memory
        x = streams if c.streams == 1 else kernels.loop_mem_norm(streams, c.streams, c.d_model)
        lat = kernels.loop_mem_norm(torch.mm(x, lm.down.t()), 1, c.loop_memory_latent,
                                    lm.lat_w, lm.lat_b)
        torch.mm(lat, lm.wkv.t(), out=kv[i])

    def _lm_inject(self, streams: torch.Tensor, kv: torch.Tensor, i: int) -> None:
        """LoopMemoryHook.inject (loop_memory.py:40-52) before loop i >= 1: every
        token attends over its endpoints of loops 0..i-1 (LatentAttention,
        mla_memory.py:66-86, no mask); streams += gate * o(attention)."""
        c, lm = self.cfg, self.w.loop_memory
        qn = kernels.loop_mem_norm(streams, c.streams, c.d_model, lm.q_ln_w, lm.q_ln_b)
        att = kernels.loop_mem_attend(torch.mm(qn, lm.wq.t()), kv, i, c.loop_memory_heads,
                                      c.loop_memory_head_dim)
        kernels.loop_mem_add(streams, c.streams, torch.mm(att, lm.wo.t()), lm.gate)

    def _head(self, streams: torch.Tensor) -> torch.Tensor:
        """mhc_collapse -> final_norm -> tied LM head (model/model.py:699-707)."""
        c = self.cfg
        sb = torch.empty(streams.shape, dtype=torch.bfloat16, device=streams.device)
        kernels.add_rmsnorm(streams, None, None, c.rms_eps, out_bf16=sb, normalize=False)
        collapsed = torch.mm(sb, self.w.collapse.t())
        h = kernels.rmsnorm_bf16(collapsed, self.w.final_norm, c.rms_eps)
        return torch.mm(h, self.w.embed.t())

    # ------------------------------------------------------------- prefill
    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor, *, state: RecurrentState | None = None,
                reset_mask: torch.Tensor | None = None, last_logits_only: bool = False,
                num_loops: int | None = None) -> HybridOutput:
        """Sequence forward (LoopedHybridMoEForCausalLM.forward, inference subset)."""
        c = self.cfg
        if input_ids.dim() != 2:
            raise ValueError("input_ids must have shape [batch, time]")
        bsz, t = input_ids.shape
        loops = c.num_loops if num_loops is None else int(num_loops)
        if state is None:
            state = RecurrentState(c, bsz, self.device)
        ids = input_ids.to(self.device)
        state.folded_rings = False  # the prefill rewrites the plain CSA value rings
        reset = None if reset_mask is None else reset_mask.to(self.device, torch.bool)
        if reset is not None and bool(reset[:, 0].any()):
            state.reset_rows(reset[:, 0])
        streams = self._embed(ids.reshape(-1))  # [N, S*D] fp32
        self._run_core(streams, state, bsz, t, reset, loops)
        state.positions.fill_(t)
        w = c.streams * c.d_model
        hs = streams.view(bsz, t, w)
        if last_logits_only:
            hs = hs[:, -1:].contiguous()
        logits = self._head(hs.reshape(-1, w)).view(bsz, -1, c.vocab_size)
        self._check_ep()
        return HybridOutput(logits, state)

    def _check_ep(self) -> None:
        """Under expert parallelism, surface a failed exchange (a peer that never
        published its rows, a malformed header) as an error after an eager call
        instead of serving wrong tokens.  Skipped while a CUDA graph is being
        captured: whoever replays it checks (ExpertParallel.check)."""
        if self.ep is not None and not torch.cuda.is_current_stream_capturing():
            self.ep.check()

    def _embed(self, ids: torch.Tensor) -> torch.Tensor:
        """Residual streams of the tokens: embed + stream_seed, [N, S*D] fp32
        (model/model.py:442-444; S = 1 without hyper-connections)."""
        c = self.cfg
        if c.streams == 1:
            return kernels.embed(ids, self.w.embed, self.w.stream_seed)
        h = kernels.embed(ids, self.w.embed, None)
        seed = self.w.stream_seed.view(1, c.streams, c.d_model)
        return (h.unsqueeze(1) + seed).reshape(h.shape[0], -1)

    @torch.no_grad()
    def run_stack(self, hidden: torch.Tensor, *, state: RecurrentState | None = None,
                  num_loops: int | None = None) -> torch.Tensor:
        """The looped recurrent core on hidden states [B,T,D] (the single-block
        workload; model/model.py:618-687 without embedding and head).  Returns
        the fp32 residual stream after the last loop."""
        c = self.cfg
        bsz, t = hidden.shape[:2]
        w = c.streams * c.d_model
        if hidden.shape[2:].numel() != w:
            raise ValueError(f"hidden must be [B, T, D] (or [B, T, S, D] with {c.streams} streams)")
        if state is None:
            state = RecurrentState(c, bsz, self.device)
        streams = hidden.to(self.device, torch.float32).reshape(bsz * t, w).clone()
        self._run_core(streams, state, bsz, t, None, c.num_loops if num_loops is None else num_loops)
        state.positions.fill_(t)
        return streams.view(hidden.shape)

    def _run_core(self, streams, state, bsz, t, reset, loops) -> None:
        c = self.cfg
        if c.mhc_streams:
            return self._run_core_mhc(streams, state, bsz, t, reset, loops)
        n, d = bsz * t, c.d_model
        normed = torch.empty(n, d, dtype=torch.bfloat16, device=self.device)
        m_bf = torch.empty_like(normed)
        m_f32 = torch.empty_like(streams)
        pending = None  # bf16 update not yet added to the residual stream
        kv = self._lm_buffer(n, loops)
        fused_router_in = self._router_in_fused()
        for i in range(loops):
            if kv is not None and i > 0:
                self._lm_inject(streams, kv, i)
            for j, blk in enumerate(self.w.blocks):
                key = state_key(i, j)
                self._add_pending(streams, pending, blk.mixer_norm, out_bf16=normed)
                if isinstance(blk.mixer, GdnBlock):
                    mixed = self._gdn_prefill(blk.mixer, normed, state, key, bsz, t, reset)
                else:
                    mixed = self._csa_prefill(blk.mixer, normed, state, key, bsz, t)
                if fused_router_in:
                    kernels.add_rmsnorm_router(streams, mixed, blk.ffn_norm, blk.moe.router_norm,
                                               c.rms_eps, out_bf16=m_bf, router_in=m_f32)
                else:
                    kernels.add_rmsnorm(streams, mixed, blk.ffn_norm, c.rms_eps, out_bf16=m_bf,
                                        out_f32=m_f32)
                pending = self._moe(blk, m_bf, m_f32, state, key, bsz, t, normed=fused_router_in)
            if kv is not None and i < loops - 1:
                self._add_pending(streams, pending, None, normalize=False)
                pending = None
                self._lm_record(streams, kv, i)
        if pending is not None:
            self._add_pending(streams, pending, None, normalize=False)

    def _mhc_write(self, streams, blk: Block, maps, pending) -> None:
        """Close a sub-layer: its output (a bf16 delta, or routed expert rows +
        plan whose per-token sum is the MoE combine) into the S streams."""
        if pending is None:
            return
        if isinstance(pending, tuple):
            kernels.mhc_write(streams, self.cfg.mhc_streams, blk.mhc, maps, pending[0], pending[1])
        else:
            kernels.mhc_write(streams, self.cfg.mhc_streams, blk.mhc, maps, pending)

    def _run_core_mhc(self, streams, state, bsz, t, reset, loops) -> None:
        """The recurrent core with hyper-connections (PhysicalBlock.forward,
        model/model.py:162-264 with self.mhc): per sub-layer a read (maps +
        LayerNorm'd weighted stream sum + the block's RMSNorm) and, after the
        sub-layer, a write of its output with the same maps."""
        c = self.cfg
        n, d, ns = bsz * t, c.d_model, c.mhc_streams
        nm = 2 * ns + ns * ns
        normed = torch.empty(n, d, dtype=torch.bfloat16, device=self.device)
        m_bf = torch.empty_like(normed)
        m_f32 = torch.empty(n, d, dtype=torch.float32, device=self.device)
        maps_mix = torch.empty(n, nm, dtype=torch.float32, device=self.device)
        maps_ffn = torch.empty_like(maps_mix)
        pending, prev = None, None
        kv = self._lm_buffer(n, loops)
        for i in range(loops):
            if kv is not None and i > 0:
                self._mhc_write(streams, prev, maps_ffn, pending)
                pending, prev = None, None
                self._lm_record(streams, kv, i - 1)
                self._lm_inject(streams, kv, i)
            for j, blk in enumerate(self.w.blocks):
                key = state_key(i, j)
                self._mhc_write(streams, prev, maps_ffn, pending)
                kernels.mhc_read(streams, ns, blk.mhc, blk.mixer_norm, c.rms_eps, c.mhc_iterations,
                                 maps_mix, out_bf16=normed)
                if isinstance(blk.mixer, GdnBlock):
                    mixed = self._gdn_prefill(blk.mixer, normed, state, key, bsz, t, reset)
                else:
                    mixed = self._csa_prefill(blk.mixer, normed, state, key, bsz, t)
                kernels.mhc_write(streams, ns, blk.mhc, maps_mix, mixed)
                kernels.mhc_read(streams, ns, blk.mhc, blk.ffn_norm, c.rms_eps, c.mhc_iterations,
                                 maps_ffn, out_bf16=m_bf, out_f32=m_f32)
                pending, prev = self._moe(blk, m_bf, m_f32, state, key, bsz, t), blk
        self._mhc_write(streams, prev, maps_ffn, pending)

    def _gdn_prefill(self, g: GdnBlock, normed, state: RecurrentState, key: str, bsz: int, t: int,
                     reset) -> torch.Tensor:
        """GatedDeltaNet.forward (gated_deltanet.py:119-276) + the block's state carry."""
        c = self.cfg
        proj = torch.mm(normed, g.w_in.t())
        kernels.gdn_activate(proj, c.gdn_heads, c.gdn_key_dim, c.gdn_value_dim, g.beta_bias)
        q, k, v, gate, beta = self._gdn_views(proj.view(bsz, t, -1), (bsz, t))
        o = kernels.gdn_prefill(q, k, v, gate, beta, state.gdn_states[key],
                                decay_logit=g.decay_logit, reset=reset)
        y = torch.mm(o.view(bsz * t, -1), g.w_out.t())
        x3 = normed.view(bsz, t, -1)
        mixed = kernels.gdn_conv_gate(x3, y.view(bsz, t, -1), g.conv, reset=reset)
        # conv history for decode: the last three inputs (model/model.py:180-182)
        kernels.gdn_history_set(x3, state.gdn_conv_histories[key])
        return mixed.view(bsz * t, -1)

    def _csa_prefill(self, a: CsaBlock, normed, state: RecurrentState, key: str, bsz: int,
                     t: int) -> torch.Tensor:
        """CSA local branch (csa.py:35-75) with the remote branch disabled."""
        c = self.cfg
        hd = c.csa_heads * c.csa_head_dim
        proj = torch.mm(normed, a.w_in.t()).view(bsz, t, -1)
        q = proj[..., :hd].unflatten(-1, (c.csa_heads, c.csa_head_dim))
        k = proj[..., hd:2 * hd].unflatten(-1, (c.csa_heads, c.csa_head_dim))
        v = proj[..., 2 * hd:]
        local = kernels.csa_local_prefill(q, k, v, c.csa_window)
        h = torch.mm(local.view(bsz * t, -1), a.local_out.t())
        if c.csa_compression:
            # remote branch (csa.py:77-131): out(local_out(local) + remote_out(remote))
            remote, summ = kernels.csa_remote_prefill(
                normed.view(bsz, t, -1), proj[..., :hd], a.w_comp, c.csa_compression, c.csa_top_k,
                c.csa_heads, state.remote_sum[key], state.remote_pending[key])
            n = summ.shape[1]
            if n > state.remote_k[key].shape[1]:
                raise ValueError(f"{t} prompt tokens exceed the state's remote memory "
                                 f"(RecurrentState max_len {state.max_len})")
            state.remote_k[key][:, :n] = summ[..., :hd]
            state.remote_v[key][:, :n] = summ[..., hd:]
            state.remote_count[key].fill_(n)
            h.addmm_(remote.view(bsz * t, -1), a.remote_out.t())
        mixed = torch.mm(h, a.out.t())
        # ring caches for decode: token p at slot p % W (last min(T, W) tokens)
        kernels.csa_ring_write(proj[..., hd:2 * hd], proj[..., 2 * hd:], state.local_k[key],
                               state.local_v[key])
        return mixed

    # -------------------------------------------------------------- decode
    @torch.no_grad()
    def decode_step(self, input_ids: torch.Tensor, state: RecurrentState,
                    num_loops: int | None = None) -> torch.Tensor:
        logits = self._decode_step(input_ids, state, num_loops)
        self._check_ep()
        return logits

    def _persistent_for(self, state: RecurrentState):
        from .persistent import PersistentDecode
        pd = getattr(state, "_persistent", None)
        if pd is None or pd.model is not self:
            pd = PersistentDecode(self, state)
            state._persistent = pd
        return pd

    def prepare_decode(self, state: RecurrentState) -> None:
        """Work the decode path needs once per state and must not capture in a
        CUDA graph (the persistent step folds the CSA value rings a prefill left)."""
        from . import persistent
        if self.decode_persistent and persistent.supported(self, state.batch):
            self._persistent_for(state).prepare()

    def greedy_fused(self, batch: int) -> bool:
        """Whether a greedy decode step of this model samples inside the
        persistent decode launch (the LM head fused with the argmax)."""
        from . import persistent
        return self.decode_persistent and persistent.supported(self, batch)

    def decode_step_greedy(self, ids: torch.Tensor, state: RecurrentState, out_token: torch.Tensor,
                           logprob: torch.Tensor | None = None,
                           seen: torch.Tensor | None = None) -> torch.Tensor:
        """decode_step followed by greedy sampling (temperature 0, no repetition
        penalty) in one persistent launch; out_token [1] int64 receives the
        token.  Requires greedy_fused(1).  Returns the logits [1, V] fp32."""
        pd = self._persistent_for(state)
        logits = pd.step(ids.reshape(-1), out_token=out_token, logprob=logprob, seen=seen)
        if self.route_log is not None:
            self.route_log.extend(pd.route_idx[r:r + 1] for r in range(pd.route_idx.shape[0]))
        return logits

    def _decode_persist(self, ids: torch.Tensor, state: RecurrentState,
                        loops: int | None = None) -> torch.Tensor:
        pd = self._persistent_for(state)
        logits = pd.step(ids, n_loops=loops)
        if self.route_log is not None:
            rows = (loops or self.cfg.num_loops) * self.cfg.n_blocks
            self.route_log.extend(pd.route_idx[r:r + 1] for r in range(rows))
        return logits

    def _decode_step(self, input_ids: torch.Tensor, state: RecurrentState,
                     num_loops: int | None = None) -> torch.Tensor:
        """One token per row (LoopedHybridMoEForCausalLM.decode_step, model/model.py:787-915,
        with the loop output carried as in sample_standalone.py's copy).

        input_ids [B] or [B, 1] on the device.  Updates `state` in place
        (GDN states, conv histories, ring caches, positions) and returns the
        logits [B, V] (bf16).  Allocation-stable, so it can be captured in a
        CUDA graph after one warm-up call.  Per block: fused residual+norm,
        one projection GEMM, the mixer kernel(s), one output GEMM, the fused
        residual+norm+router+plan, two expert kernels; the MoE combine is
        folded into the next block's residual add.
        """
        c = self.cfg
        ids = input_ids.reshape(-1)
        bsz = ids.shape[0]
        loops = c.num_loops if num_loops is None else int(num_loops)
        d = c.d_model
        if self.decode_persistent and 1 <= loops <= c.num_loops:
            from . import persistent
            if persistent.supported(self, bsz):
                return self._decode_persist(ids, state, loops)
        if getattr(state, "folded_rings", False):
            raise RuntimeError("this state is advanced by the persistent decode step (its CSA "
                               "value rings are folded); continue with decode_persistent=True "
                               "or start again with a prefill")
        if c.mhc_streams:
            return self._decode_mhc(ids, state, loops)
        csa_in = 2 * d if c.csa_compression else d  # input width of the CSA output projection
        if self.decode_fused and not c.router_context and kernels.decode_fused_supported(
                bsz, d, c.moe_experts, c.moe_top_k, c.gdn_heads * c.gdn_value_dim, csa_in):
            return self._decode_fused(ids, state, loops)
        fused_router = (not c.router_context
                        and kernels.route_fused_supported(bsz, c.moe_experts, c.moe_top_k, d))
        # 128-row tiles for the grouped expert GEMMs at a few rows per expert
        tile_m = 128
        streams = kernels.embed(ids, self.w.embed, self.w.stream_seed)
        normed = torch.empty(bsz, d, dtype=torch.bfloat16, device=self.device)
        m_bf = torch.empty_like(normed)
        m_f32 = torch.empty_like(streams)
        y_rows, plan = None, None
        kv = self._lm_buffer(bsz, loops)
        for i in range(loops):
            if kv is not None and i > 0:
                kernels.add_rmsnorm_routed(streams, y_rows, plan, None, c.rms_eps, normalize=False)
                y_rows, plan = None, None
                self._lm_record(streams, kv, i - 1)
                self._lm_inject(streams, kv, i)
            for j, blk in enumerate(self.w.blocks):
                key = state_key(i, j)
                if y_rows is None:
                    kernels.add_rmsnorm(streams, None, blk.mixer_norm, c.rms_eps, out_bf16=normed)
                else:
                    kernels.add_rmsnorm_routed(streams, y_rows, plan, blk.mixer_norm, c.rms_eps,
                                               out_bf16=normed)
                if isinstance(blk.mixer, GdnBlock):
                    mixed = self._gdn_step(blk.mixer, normed, state, key, bsz)
                else:
                    mixed = self._csa_step(blk.mixer, normed, state, key, bsz)
                if fused_router:
                    plan = kernels.route_fused(streams, mixed, blk.ffn_norm, blk.moe.router_norm,
                                               blk.moe.router, c.moe_top_k, c.rms_eps, m_bf,
                                               tile_m=tile_m)
                else:
                    kernels.add_rmsnorm(streams, mixed, blk.ffn_norm, c.rms_eps, out_bf16=m_bf,
                                        out_f32=m_f32)
                    logits = self._router_logits(blk, m_f32, state, key, bsz, 1, step=True)
                    plan = kernels.route(logits, c.moe_top_k, tile_m=tile_m)
                y_rows, plan = self._experts(blk, m_bf, plan)
        return self._decode_head(streams, y_rows, plan, state)

    def _experts(self, blk: Block, m_bf: torch.Tensor, plan: kernels.RoutePlan):
        """Routed (and shared) expert rows and the plan that combines them
        (prefill and decode).  Shared experts (moe.py:185-198, :221-234) are
        plan experts E..E+S-1 that every token is routed to with probability
        1/sqrt(S), stacked after the routed experts in w13 / w2."""
        if self.route_log is not None:
            self.route_log.append(plan.topk_idx)
        if self.cfg.moe_shared:
            plan = kernels.plan_append_shared(plan, self.cfg.moe_shared)
        if self.ep is not None:
            res = self.ep.run(m_bf, plan, blk.moe.w13, blk.moe.w2, path=self.expert_path)
            return res.y_rows, res.plan_for_combine(plan)
        return kernels.moe_experts_rows(m_bf, plan, blk.moe.w13, blk.moe.w2,
                                        path=self.expert_path), plan

    def _decode_head(self, streams, y_rows, plan, state: RecurrentState) -> torch.Tensor:
        c = self.cfg
        bsz, d = streams.shape
        sb = torch.empty(bsz, d, dtype=torch.bfloat16, device=self.device)
        kernels.add_rmsnorm_routed(streams, y_rows, plan, None, c.rms_eps, out_bf16=sb,
                                   normalize=False)
        collapsed = torch.mm(sb, self.w.collapse.t())
        h = kernels.rmsnorm_bf16(collapsed, self.w.final_norm, c.rms_eps)
        logits = torch.mm(h, self.w.embed.t())
        state.positions.add_(1)
        return logits

    def _decode_mhc(self, ids: torch.Tensor, state: RecurrentState, loops: int) -> torch.Tensor:
        """decode_step with hyper-connections (PhysicalBlock.forward_step,
        model/model.py:266-376 with self.mhc): the read / write pairs of the
        prefill core around the mixer step kernels and the routed experts."""
        c = self.cfg
        bsz, d, ns = ids.shape[0], c.d_model, c.mhc_streams
        nm = 2 * ns + ns * ns
        streams = self._embed(ids)
        normed = torch.empty(bsz, d, dtype=torch.bfloat16, device=self.device)
        m_bf = torch.empty_like(normed)
        m_f32 = torch.empty(bsz, d, dtype=torch.float32, device=self.device)
        maps_mix = torch.empty(bsz, nm, dtype=torch.float32, device=self.device)
        maps_ffn = torch.empty_like(maps_mix)
        pending, prev = None, None
        kv = self._lm_buffer(bsz, loops)
        for i in range(loops):
            if kv is not None and i > 0:
                self._mhc_write(streams, prev, maps_ffn, pending)
                pending, prev = None, None
                self._lm_record(streams, kv, i - 1)
                self._lm_inject(streams, kv, i)
            for j, blk in enumerate(self.w.blocks):
                key = state_key(i, j)
                self._mhc_write(streams, prev, maps_ffn, pending)
                kernels.mhc_read(streams, ns, blk.mhc, blk.mixer_norm, c.rms_eps, c.mhc_iterations,
                                 maps_mix, out_bf16=normed)
                if isinstance(blk.mixer, GdnBlock):
                    mixed = self._gdn_step(blk.mixer, normed, state, key, bsz)
                else:
                    mixed = self._csa_step(blk.mixer, normed, state, key, bsz)
                kernels.mhc_write(streams, ns, blk.mhc, maps_mix, mixed)
                kernels.mhc_read(streams, ns, blk.mhc, blk.ffn_norm, c.rms_eps, c.mhc_iterations,
                                 maps_ffn, out_bf16=m_bf, out_f32=m_f32)
                logits = self._router_logits(blk, m_f32, state, key, bsz, 1, step=True)
                plan = kernels.route(logits, c.moe_top_k, tile_m=128)
                pending, prev = self._experts(blk, m_bf, plan), blk
        self._mhc_write(streams, prev, maps_ffn, pending)
        h = kernels.rmsnorm_bf16(torch.mm(streams.to(torch.bfloat16), self.w.collapse.t()),
                                 self.w.final_norm, c.rms_eps)
        state.positions.add_(1)
        return torch.mm(h, self.w.embed.t())

    def _decode_fused(self, ids: torch.Tensor, state: RecurrentState, loops: int) -> torch.Tensor:
        """decode_step on the fused small-batch kernels: per block [A] residual
        add + norm + input projection, the mixer kernel, [C] output projection
        (+ conv gate) + residual + norms + router + plan, the two expert
        kernels.  The residual stream alternates between two buffers because
        every CTA of [A] reads the old value while one CTA writes the new."""
        c = self.cfg
        bsz, d = ids.shape[0], c.d_model
        cur = kernels.embed(ids, self.w.embed, self.w.stream_seed)
        nxt = torch.empty_like(cur)
        normed = torch.empty(bsz, d, dtype=torch.bfloat16, device=self.device)
        m_bf = torch.empty_like(normed)
        y_rows, plan = None, None
        kv = self._lm_buffer(bsz, loops)
        for i in range(loops):
            if kv is not None and i > 0:
                kernels.add_rmsnorm_routed(cur, y_rows, plan, None, c.rms_eps, normalize=False)
                y_rows, plan = None, None
                self._lm_record(cur, kv, i - 1)
                self._lm_inject(cur, kv, i)
            for j, blk in enumerate(self.w.blocks):
                key = state_key(i, j)
                mix = blk.mixer
                proj = torch.empty(bsz, mix.w_in.shape[0], dtype=torch.bfloat16, device=self.device)
                kernels.decode_norm_gemv(cur, y_rows, plan, blk.mixer_norm, c.rms_eps, mix.w_in,
                                         proj, nxt, normed)
                cur, nxt = nxt, cur
                router = (cur, blk.ffn_norm, blk.moe.router_folded, c.moe_top_k, c.rms_eps, m_bf,
                          self._counter)
                if isinstance(mix, GdnBlock):
                    q, k, v, gate, beta = self._gdn_views(proj, (bsz,))
                    o = kernels.gdn_step(q, k, v, gate, beta, state.gdn_states[key],
                                         decay_logit=mix.decay_logit, raw_inputs=True,
                                         beta_bias=mix.beta_bias)
                    plan = kernels.decode_out_router(
                        o.view(bsz, -1), mix.w_out, *router, conv_w=mix.conv, normed=normed,
                        history=state.gdn_conv_histories[key], tile_m=128)
                else:
                    attn = self._csa_mix_step(mix, proj, normed, state, key, bsz)
                    plan = kernels.decode_out_router(attn, mix.w_o, *router, tile_m=128)
                y_rows, plan = self._experts(blk, m_bf, plan)
        return self._decode_head(cur, y_rows, plan, state)

    def _gdn_step(self, g: GdnBlock, normed, state: RecurrentState, key: str, bsz: int):
        c = self.cfg
        proj = torch.mm(normed, g.w_in.t())
        q, k, v, gate, beta = self._gdn_views(proj, (bsz,))
        o = kernels.gdn_step(q, k, v, gate, beta, state.gdn_states[key], decay_logit=g.decay_logit,
                             raw_inputs=True, beta_bias=g.beta_bias)
        y = torch.mm(o.view(bsz, -1), g.w_out.t())
        return kernels.gdn_conv_gate(normed.view(bsz, 1, -1), y.view(bsz, 1, -1), g.conv,
                                     history=state.gdn_conv_histories[key],
                                     roll_history=True).view(bsz, -1)

    def _csa_step(self, a: CsaBlock, normed, state: RecurrentState, key: str, bsz: int):
        c = self.cfg
        hd = c.csa_heads * c.csa_head_dim
        proj = torch.mm(normed, a.w_in.t())
        return torch.mm(self._csa_mix_step(a, proj, normed, state, key, bsz), a.w_o.t())

    def _csa_mix_step(self, a: CsaBlock, proj, normed, state: RecurrentState, key: str,
                      bsz: int):
        """The CSA decode step's attention outputs: local [B, D], or with the
        remote branch [local | remote] [B, 2D] (the input of w_o; csa.py:172-256)."""
        c = self.cfg
        hd, d = c.csa_heads * c.csa_head_dim, c.d_model
        width = 2 * d if c.csa_compression else d
        mix = torch.empty(bsz, width, dtype=torch.bfloat16, device=self.device)
        kernels.csa_local_decode(proj[:, :hd], proj[:, hd:2 * hd], proj[:, 2 * hd:],
                                 state.local_k[key], state.local_v[key], state.positions,
                                 c.csa_heads, out=mix[:, :d])
        if c.csa_compression:
            kernels.csa_remote_step(normed, proj[:, :hd], a.w_comp, c.csa_compression, c.csa_top_k, c.csa_heads,
                                    state.remote_k[key], state.remote_v[key],
                                    state.remote_count[key], state.remote_sum[key],
                                    state.remote_pending[key], mix[:, d:])
        return mix


class GreedyDecoder:
    """Decode loop with the whole step (model + sampler) captured in one CUDA graph.

    The sampled token feeds the next step's embedding on the device; `step()`
    replays the graph once per token (the role of _CudaGraphDecoder,
    sample_standalone.py:4562-4794).
    """

    def __init__(self, model: LoopedHybridModel, state: RecurrentState, *, use_graph: bool = True,
                 temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0,
                 repetition_penalty: float = 1.0):
        self.model, self.state = model, state
        self.bsz = state.batch
        dev = model.device
        self.tokens = torch.zeros(self.bsz, dtype=torch.int64, device=dev)
        self.uniforms = torch.zeros(self.bsz, dtype=torch.float32, device=dev)
        v = model.cfg.vocab_size
        self.seen = torch.zeros(self.bsz, (v + 31) // 32, dtype=torch.int32, device=dev)
        self.sampling = dict(temperature=temperature, top_k=top_k, top_p=top_p,
                             repetition_penalty=repetition_penalty)
        self.graph = None
        self.io_graph = None
        self.use_graph = use_graph
        self.logprob = None
        # pinned host buffers of step_host (allocated on its first call)
        self.host_in = self.host_out = self.host_lp = None
        # fp32 logits [B, V] of the last step (in graph mode the graph's own
        # output buffer, rewritten by every replay)
        self.logits = None

    def _body(self):
        s = self.sampling
        if (s["temperature"] <= 1e-4 and s["repetition_penalty"] == 1.0
                and self.model.greedy_fused(self.bsz)):
            # greedy: the LM head and the argmax run inside the decode launch
            if self.logprob is None:
                self.logprob = torch.zeros(self.bsz, dtype=torch.float32, device=self.tokens.device)
            logits = self.model.decode_step_greedy(self.tokens, self.state, self.tokens,
                                                   self.logprob, self.seen.view(-1))
            self.logits = logits
            return logits
        logits = self.model.decode_step(self.tokens, self.state).float()
        tok, lp = kernels.sample(logits, seen=self.seen, uniforms=self.uniforms, update_seen=True,
                                 out=self.tokens, **self.sampling)
        self.logprob = lp
        self.logits = logits
        return logits

    def prime(self, first_tokens: torch.Tensor) -> None:
        self.tokens.copy_(first_tokens.reshape(-1))

    def capture(self) -> None:
        """Warm up once (eager) on a copy of the state, then capture the step."""
        saved = self.state.state_dict()
        tok0 = self.tokens.clone()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._body()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.state.load_state_dict(saved)
        self.model.prepare_decode(self.state)
        self.tokens.copy_(tok0)
        self.seen.zero_()
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._body()
        torch.cuda.synchronize()

    def step(self) -> torch.Tensor:
        if self.use_graph:
            if self.graph is None:
                self.capture()
            self.graph.replay()
        else:
            self._body()
        return self.tokens

    def step_host(self) -> tuple[torch.Tensor, torch.Tensor]:
        """One step with the host round trip inside the graph: the tokens in
        self.host_in (pinned, [B] int64) go to the device, the step runs, and the
        sampled tokens and their log-probabilities come back into self.host_out
        and self.host_lp (pinned) -- one graph submission per step; the caller
        synchronizes the stream before reading them.  Call step() once first (it
        captures the step); the first step_host() call captures this graph."""
        if self.graph is None:
            raise RuntimeError("call step() once before step_host()")
        if self.io_graph is None:
            self.host_in = torch.empty(self.bsz, dtype=torch.int64).pin_memory()
            self.host_out = torch.empty(self.bsz, dtype=torch.int64).pin_memory()
            self.host_lp = torch.empty(self.bsz, dtype=torch.float32).pin_memory()
            self.host_in.copy_(self.tokens.cpu())
            torch.cuda.synchronize()
            self.io_graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.io_graph):
                self.tokens.copy_(self.host_in, non_blocking=True)
                self._body()
                self.host_out.copy_(self.tokens, non_blocking=True)
                self.host_lp.copy_(self.logprob, non_blocking=True)
            torch.cuda.synchronize()
        self.io_graph.replay()
        return self.host_out, self.host_lp


class StackGraph:
    """The looped recurrent core on hidden states of a fixed shape [batch, seq,
    D] (run_stack: model/model.py:618-687 without embedding and head) captured
    in one CUDA graph.  At a few hundred tokens the eager core is bound by the
    host cost of its launches; a replay issues them at once.  Each replay
    starts from a zeroed RecurrentState (zeroed inside the graph) and returns
    the graph's own fp32 output stream, which the next replay overwrites."""

    def __init__(self, model: LoopedHybridModel, batch: int, seq: int,
                 num_loops: int | None = None):
        dev = model.device
        self.model, self.num_loops = model, num_loops
        w = model.cfg.streams * model.cfg.d_model
        self.hidden = torch.zeros(batch, seq, w, dtype=torch.float32, device=dev)
        self.state = RecurrentState(model.cfg, batch, dev)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):  # warm-up: workspaces and one-time attributes
            self._body()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = self._body()
        torch.cuda.synchronize()

    def _body(self) -> torch.Tensor:
        self.state.zero_()
        return self.model.run_stack(self.hidden, state=self.state, num_loops=self.num_loops)

    def run(self, hidden: torch.Tensor) -> torch.Tensor:
        """The core on `hidden` [batch, seq, D] (device or host): copies it into
        the graph's input buffer and replays."""
        if tuple(hidden.shape) != tuple(self.hidden.shape):
            raise ValueError(f"this graph was captured for hidden states of shape "
                             f"{tuple(self.hidden.shape)}")
        self.hidden.copy_(hidden, non_blocking=True)
        self.graph.replay()
        return self.out


class PrefillGraph:
    """A prompt forward of fixed shape [batch, seq] captured in one CUDA graph.

    The eager forward issues a few hundred kernel launches per prompt and, at
    short prompts, is bound by their host-side cost (the c2 512-token prompt:
    ~7.4 ms eager for ~3.5 ms of kernels); a replay issues them at once.  Each
    replay starts from a zeroed RecurrentState (zeroed inside the graph) and
    returns the graph's own outputs -- the last-position logits [B, 1, V] and
    the state the prompt leaves -- which the next replay overwrites: hand the
    state to a decoder (or copy it) before running another prompt.
    """

    def __init__(self, model: LoopedHybridModel, batch: int, seq: int,
                 num_loops: int | None = None):
        dev = model.device
        self.model, self.num_loops = model, num_loops
        self.ids = torch.zeros(batch, seq, dtype=torch.int64, device=dev)
        self.state = RecurrentState(model.cfg, batch, dev)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):  # warm-up: workspaces and one-time attributes
            self._body()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = self._body()
        torch.cuda.synchronize()

    def _body(self) -> HybridOutput:
        self.state.zero_()
        return self.model.forward(self.ids, state=self.state, last_logits_only=True,
                                  num_loops=self.num_loops)

    def run(self, input_ids: torch.Tensor) -> HybridOutput:
        """Prefill `input_ids` [batch, seq] (device or host): copies the ids
        into the graph's input buffer and replays."""
        if tuple(input_ids.shape) != tuple(self.ids.shape):
            raise ValueError(f"this graph was captured for ids of shape {tuple(self.ids.shape)}")
        self.ids.copy_(input_ids, non_blocking=True)
        self.graph.replay()
        self.state.folded_rings = False
        return self.out
