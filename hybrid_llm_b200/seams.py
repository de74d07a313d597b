"""Drop-in replacements for the reference's kernel hooks (its plugin API).

The reference model (StillPillWill/Hybrid_LLM, ``model/``) calls its
accelerated kernels through module-level hooks and availability flags; the
functions below have the same signatures and semantics and run the llmyb
CUDA kernels instead:

=============================================  ==========================================
reference hook (file:line)                     replacement
=============================================  ==========================================
model.layers.moe._triton_moe_dispatch          :func:`triton_moe_dispatch`
  (moe.py:16-25, called :163-167)
model.layers.gated_deltanet._triton_gdn_scan   :func:`triton_gdn_scan`
  (gated_deltanet.py:30-39, called :216-235)
model.layers.gated_deltanet._triton_gdn_step   :func:`triton_gdn_step`
  (called :179-187; updates ``state`` in place)
runpod.kernels.triton_banded_attention.        :func:`triton_banded_local_attention`
  triton_banded_local_attention (csa.py:44-53,
  sample_standalone.py:390-409)
(no hook) topk + softmax, context_router.py:73  :func:`router_topk`
_sample_next_token (sample_standalone.py:5383)  :func:`sample_next_token`
=============================================  ==========================================

:func:`install` patches the hooks into already-imported reference modules.
The hooks only fire for CUDA tensors (the reference checks ``is_cuda``); a
CPU tensor passed here raises instead of falling back.  The kernels compute
in bf16 with fp32 accumulation (fp32 inputs are rounded to bf16 on entry,
outputs are returned in the input dtype), the GDN state stays fp32.
"""
from __future__ import annotations

import sys
import weakref
from typing import Any

import torch

from . import kernels

# ------------------------------------------------------------------- MoE
_w13_cache: dict[tuple, tuple[weakref.ref, torch.Tensor]] = {}


def _packed_w13(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    key = (w_gate.data_ptr(), w_up.data_ptr(), tuple(w_gate.shape), w_gate.dtype,
           w_gate._version, w_up._version)
    hit = _w13_cache.get(key)
    if hit is not None and hit[0]() is not None:
        return hit[1]
    packed = kernels.pack_w13(w_gate, w_up)
    _w13_cache.clear()  # the reference keeps one stacked copy per module; so do we
    _w13_cache[key] = (weakref.ref(w_gate), packed)
    return packed


def triton_moe_dispatch(flat: torch.Tensor, indices: torch.Tensor, probabilities: torch.Tensor,
                        routed_experts: int, w_gate: torch.Tensor, w_up: torch.Tensor,
                        w_down: torch.Tensor) -> torch.Tensor:
    """Routed SwiGLU experts for top-k routes (moe.py:29-82 semantics).

    flat [N, D]; indices [N, k] int64; probabilities [N, k]; w_gate/w_up
    [E, F, D]; w_down [E, D, F].  Returns [N, D] in flat's dtype.
    """
    plan = kernels.moe_plan(indices, probabilities, int(routed_experts))
    x = flat.to(torch.bfloat16)
    out = kernels.moe_grouped(x, plan, _packed_w13(w_gate, w_up), w_down.to(torch.bfloat16))
    return out.to(flat.dtype)


def router_topk(route_logits: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(top_indices int64, probabilities fp32) = topk(logits.float(), k) + softmax
    (context_router.py:73-74); ties are broken by the lower expert index."""
    lead = route_logits.shape[:-1]
    idx, prob = kernels.router_topk(route_logits.reshape(-1, route_logits.shape[-1]).float(), k)
    return idx.view(*lead, k), prob.view(*lead, k)


# ------------------------------------------------------------------- GDN
def _bf(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)


def triton_gdn_scan(q, k, v, beta, gate, reset, decay_logit, state):
    """Chunked GDN scan (gated_deltanet.py:140-149 semantics).

    q, k [B,T,H,K] (L2-normalised); v, gate [B,T,H,V]; beta [B,T,H,1]
    (sigmoided); reset [B,T] bool; decay_logit [H]; state [B,H,K,V].
    Returns (out [B,T,H,V] in q's dtype, final state [B,H,K,V] fp32).
    """
    final = state.to(torch.float32).clone().contiguous()
    out = kernels.gdn_prefill(_bf(q).contiguous(), _bf(k).contiguous(), _bf(v).contiguous(),
                              _bf(gate).contiguous(), _bf(beta[..., 0]).contiguous(), final,
                              decay_logit=decay_logit.float(), reset=reset)
    return out.to(q.dtype), final


def triton_gdn_step(q, k, v, beta, gate, reset, decay_logit, state):
    """One-token GDN update; updates ``state`` in place and returns it."""
    b, t, h, kd = q.shape
    if t != 1:
        raise ValueError("triton_gdn_step expects one token per row")
    st = state if (state.dtype == torch.float32 and state.is_contiguous()) else \
        state.to(torch.float32).contiguous()
    out = kernels.gdn_step(_bf(q[:, 0]).contiguous(), _bf(k[:, 0]).contiguous(),
                           _bf(v[:, 0]).contiguous(), _bf(gate[:, 0]).contiguous(),
                           _bf(beta[:, 0, :, 0]).contiguous(), st,
                           decay_logit=decay_logit.float(),
                           reset=None if reset is None else reset[:, 0])
    if st is not state:
        state.copy_(st)
    return out.unsqueeze(1).to(q.dtype), state


# ----------------------------------------------------- banded attention
def triton_banded_local_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                  window_size: int = 128) -> torch.Tensor:
    """Per-head causal window attention (sample_standalone.py:390-409 contract).

    q, k [B,T,H,D] with D in {64, 128}; v [B,T,H,D] or one shared stream
    [B,T,1,Dv] (CSA).  Returns [B,T,H,Dv].  For the CSA caller, which takes
    ``.mean(2)`` of the result, :func:`csa_local_attention` computes the
    mean directly and is much cheaper.
    """
    qb, kb, vb = _bf(q).contiguous(), _bf(k).contiguous(), _bf(v).contiguous()
    d = q.shape[-1]
    if vb.shape[2] == q.shape[2] or vb.shape[-1] == d:
        return kernels.banded_attention(qb, kb, vb, int(window_size)).to(q.dtype)
    # shared value stream wider than a head: one head-width slice at a time
    parts = [kernels.banded_attention(qb, kb, vb[..., c:c + d].contiguous(), int(window_size))
             for c in range(0, vb.shape[-1], d)]
    return torch.cat(parts, dim=-1).to(q.dtype)


def csa_local_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                        window_size: int) -> torch.Tensor:
    """CSA local branch in one call: mean over heads of the per-head window
    attention on the shared value stream (csa.py:54-75).  q, k [B,T,H,Dh];
    v [B,T,D] -> [B,T,D]."""
    return kernels.csa_local_prefill(_bf(q), _bf(k), _bf(v), int(window_size)).to(q.dtype)


# ------------------------------------------------------------- sampling
def sample_next_token(logits: torch.Tensor, generated: list[int], *, temp: float, top_k: int,
                      top_p: float, rep: float) -> tuple[torch.Tensor, torch.Tensor]:
    """_sample_next_token (sample_standalone.py:5383-5423): returns
    (next_tok [B,1] int64, raw log-probability of that token [B,1])."""
    lg = logits.float().contiguous()
    rows = lg.shape[0]
    seen = kernels.seen_bitmask([generated] * rows, lg.shape[1], lg.device) if rep != 1.0 else None
    tok, lp = kernels.sample(lg, temperature=temp, top_k=top_k, top_p=top_p,
                             repetition_penalty=rep, seen=seen)
    return tok.view(rows, 1), lp.view(rows, 1)


# -------------------------------------------------------------- install
def install(moe_module: Any = None, gdn_module: Any = None, banded_module: Any = None) -> None:
    """Point the reference's hooks at the llmyb kernels.

    Each argument is the imported reference module (or None to look it up in
    ``sys.modules``): ``model.layers.moe``, ``model.layers.gated_deltanet``,
    ``runpod.kernels.triton_banded_attention``.  Modules that are absent are
    skipped.
    """
    moe_module = moe_module or sys.modules.get("model.layers.moe")
    gdn_module = gdn_module or sys.modules.get("model.layers.gated_deltanet")
    banded_module = banded_module or sys.modules.get("runpod.kernels.triton_banded_attention")
    if moe_module is not None:
        moe_module._triton_moe_dispatch = triton_moe_dispatch
        moe_module._triton_available = True
    if gdn_module is not None:
        gdn_module._triton_gdn_scan = triton_gdn_scan
        gdn_module._triton_gdn_step = triton_gdn_step
        gdn_module._triton_gdn_available = True
        gdn_module._fused_gdn_scan = None
        gdn_module._fused_gdn_step = None
    if banded_module is not None:
        banded_module.triton_banded_local_attention = triton_banded_local_attention
