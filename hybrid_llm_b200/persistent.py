"""Batch-1 decode step as one persistent launch (llmyb_decode_persistent).

Host side of csrc/decode_persistent.cu: the ctypes mirror of the C structs
in include/llmyb.h, the weights the kernel reads (the CSA value rows folded
with the output projection), the folded value rings, the scratch buffers,
and the step itself.  The kernel computes the decode step of
LoopedHybridModel.decode_step (model/model.py:787-915) for one row of the
served subset: one plain residual stream, CSA without the remote branch,
GDN, routed experts, no loop memory.

The CSA output projection out(local_out(.)) is linear and applied after the
head-averaged attention sum, so out = sum_j p_j (W_o v_j) with W_o =
out . local_out: the kernel's input projection produces W_o W_v x for the
value rows and the ring keeps those folded values (`RecurrentState.local_vo`),
so the attention output is the block output.  `prepare()` folds the plain
rings a prefill left (local_v) once; from then on the persistent step keeps
local_vo and the plain rings fall behind, so a state stays with this path
(`RecurrentState.folded_rings`) until the next prefill.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _native, kernels
from .config import HybridConfig
from .state import RecurrentState, state_key
from .weights import CsaBlock, GdnBlock


class PBlock(C.Structure):
    _fields_ = [("kind", C.c_int32), ("rows", C.c_int32), ("mixer_norm", C.c_void_p),
                ("ffn_norm", C.c_void_p), ("router_fold", C.c_void_p), ("w_in", C.c_void_p),
                ("beta_bias", C.c_void_p), ("decay_logit", C.c_void_p), ("w_out", C.c_void_p),
                ("conv", C.c_void_p), ("w13", C.c_void_p), ("w2", C.c_void_p)]


class PLayer(C.Structure):
    _fields_ = [("ring_k", C.c_void_p), ("ring_v", C.c_void_p), ("gdn_state", C.c_void_p),
                ("conv_hist", C.c_void_p)]


class PDecode(C.Structure):
    _fields_ = [("d_model", C.c_int32), ("n_blocks", C.c_int32), ("n_loops", C.c_int32),
                ("vocab", C.c_int32), ("csa_heads", C.c_int32), ("csa_head_dim", C.c_int32),
                ("window", C.c_int32), ("gdn_heads", C.c_int32), ("gdn_dim", C.c_int32),
                ("n_experts", C.c_int32), ("top_k", C.c_int32), ("ffn", C.c_int32),
                ("eps", C.c_float), ("grid", C.c_int32), ("blocks", C.c_void_p),
                ("layers", C.c_void_p), ("embed", C.c_void_p), ("stream_seed", C.c_void_p),
                ("collapse", C.c_void_p), ("final_norm", C.c_void_p), ("token", C.c_void_p),
                ("positions", C.c_void_p), ("x", C.c_void_p), ("proj", C.c_void_p),
                ("normed", C.c_void_p), ("scores", C.c_void_p), ("stats", C.c_void_p),
                ("mix", C.c_void_p), ("partials", C.c_void_p), ("hbuf", C.c_void_p),
                ("ybuf", C.c_void_p), ("collapsed", C.c_void_p), ("route_idx", C.c_void_p),
                ("route_prob", C.c_void_p), ("logits", C.c_void_p), ("bar", C.c_void_p),
                ("status", C.c_void_p), ("trace", C.c_void_p), ("out_token", C.c_void_p),
                ("out_logprob", C.c_void_p), ("seen", C.c_void_p), ("head_part", C.c_void_p),
                ("skip_head", C.c_int32)]


def supported(model, batch: int) -> bool:
    """Whether the persistent step serves this model at this batch size."""
    c: HybridConfig = model.cfg
    if batch != 1 or model.ep is not None or model.expert_path != "auto":
        return False
    if c.mhc_streams or c.router_context or c.csa_compression or c.moe_shared or c.loop_memory:
        return False
    d = c.d_model
    has_csa = any(b.kind == "csa" for b in model.w.blocks)
    has_gdn = any(b.kind == "gdn" for b in model.w.blocks)
    if d % 8 or d > 1024 or c.moe_hidden % 128 or c.moe_hidden > 2048:
        return False
    if c.moe_experts > 64 or c.moe_top_k > 8 or c.vocab_size >= 2 ** 31:
        return False
    if has_csa and (c.csa_head_dim != 64 or c.csa_heads > 16 or c.csa_window > 1024
                    or c.csa_heads * c.csa_head_dim > 1024):
        return False
    if has_gdn and (c.gdn_key_dim != 64 or c.gdn_value_dim != 64
                    or c.gdn_heads * 64 > 1024):
        return False
    grid = grid_size()
    if grid <= 0 or d > grid * 16 or (has_csa and (d // 8 > grid or -(-c.csa_window // 16) > grid)):
        return False
    if has_gdn and c.gdn_heads * 2 > grid:
        return False
    rows = max(b.mixer.w_in.shape[0] for b in model.w.blocks)
    return rows <= 2 * grid * 16


_grid: int | None = None


def grid_size() -> int:
    global _grid
    if _grid is None:
        _grid = int(_native.lib().llmyb_decode_persistent_grid())
    return _grid


def fold_csa_weights(blk: CsaBlock, cfg: HybridConfig) -> torch.Tensor:
    """[Wq; Wk; W_o W_v] (bf16, the product in fp32): the input projection whose
    value rows produce the folded values the persistent step caches."""
    hd = cfg.csa_heads * cfg.csa_head_dim
    wv = blk.w_in[2 * hd:].float()
    return torch.cat([blk.w_in[:2 * hd], (blk.w_o.float() @ wv).to(torch.bfloat16)]).contiguous()


class PersistentDecode:
    """Tables and scratch of the persistent step for one (model, state) pair."""

    def __init__(self, model, state: RecurrentState):
        c = model.cfg
        if not supported(model, state.batch):
            raise ValueError("the persistent decode step does not serve this model / batch")
        self.model, self.state = model, state
        dev = model.device
        self.grid = grid_size()
        d, e, k, f = c.d_model, c.moe_experts, c.moe_top_k, c.moe_hidden
        nb, nl = c.n_blocks, c.num_loops
        keep = []   # tensors the device tables point at
        blocks = (PBlock * nb)()
        for j, b in enumerate(model.w.blocks):
            pb = blocks[j]
            pb.mixer_norm, pb.ffn_norm = b.mixer_norm.data_ptr(), b.ffn_norm.data_ptr()
            pb.router_fold = b.moe.router_folded.data_ptr()
            pb.w13, pb.w2 = b.moe.w13.data_ptr(), b.moe.w2.data_ptr()
            if isinstance(b.mixer, CsaBlock):
                w_in = fold_csa_weights(b.mixer, c)
                keep.append(w_in)
                pb.kind, pb.rows, pb.w_in = 0, w_in.shape[0], w_in.data_ptr()
            else:
                g: GdnBlock = b.mixer
                pb.kind, pb.rows, pb.w_in = 1, g.w_in.shape[0], g.w_in.data_ptr()
                pb.beta_bias, pb.decay_logit = g.beta_bias.data_ptr(), g.decay_logit.data_ptr()
                pb.w_out, pb.conv = g.w_out.data_ptr(), g.conv.data_ptr()
        layers = (PLayer * (nb * nl))()
        for i in range(nl):
            for j in range(nb):
                key, pl = state_key(i, j), layers[i * nb + j]
                if c.block_kind(j) == "csa":
                    if key not in state.local_vo:
                        state.local_vo[key] = torch.zeros_like(state.local_v[key])
                    pl.ring_k = state.local_k[key].data_ptr()
                    pl.ring_v = state.local_vo[key].data_ptr()
                else:
                    pl.gdn_state = state.gdn_states[key].data_ptr()
                    pl.conv_hist = state.gdn_conv_histories[key].data_ptr()
        u8 = dict(dtype=torch.uint8, device=dev)
        self._blocks = torch.frombuffer(bytearray(bytes(blocks)), dtype=torch.uint8).to(dev)
        self._layers = torch.frombuffer(bytearray(bytes(layers)), dtype=torch.uint8).to(dev)
        self._keep = keep
        f32 = dict(dtype=torch.float32, device=dev)
        bf = dict(dtype=torch.bfloat16, device=dev)
        hc = c.csa_heads
        rows = max(b.mixer.w_in.shape[0] for b in model.w.blocks)
        self.token = torch.zeros(1, dtype=torch.int64, device=dev)
        self.x = torch.zeros(2, d, **f32)
        self.proj = torch.zeros(rows, **bf)
        self.normed = torch.zeros(d, **bf)
        self.scores = torch.zeros(max(hc, 1), max(c.csa_window, 1), **f32)
        self.stats = torch.zeros(max(hc, 1), self.grid, 2, **f32)
        self.mix = torch.zeros(max(d, c.gdn_heads * c.gdn_value_dim), **bf)
        self.partials = torch.zeros(2 + e, self.grid, **f32)
        self.hbuf = torch.zeros(k, f, **bf)
        self.ybuf = torch.zeros(k, d, **bf)
        self.collapsed = torch.zeros(d, **bf)
        self.route_idx = torch.zeros(nl * nb, k, dtype=torch.int32, device=dev)
        self.route_prob = torch.zeros(nl * nb, k, **f32)
        self.logits = torch.zeros(1, c.vocab_size, **f32)
        self.bar = torch.zeros(2, dtype=torch.int32, device=dev)
        self.head_part = torch.zeros(self.grid, 4, **f32)
        del u8
        p = PDecode()
        p.d_model, p.n_blocks, p.n_loops, p.vocab = d, nb, nl, c.vocab_size
        has_csa = any(b.kind == "csa" for b in model.w.blocks)
        has_gdn = any(b.kind == "gdn" for b in model.w.blocks)
        p.csa_heads = hc if has_csa else 0
        p.csa_head_dim, p.window = c.csa_head_dim, c.csa_window
        p.gdn_heads = c.gdn_heads if has_gdn else 0
        p.gdn_dim = c.gdn_key_dim
        p.n_experts, p.top_k, p.ffn, p.eps, p.grid = e, k, f, c.rms_eps, self.grid
        p.blocks, p.layers = self._blocks.data_ptr(), self._layers.data_ptr()
        w = model.w
        p.embed, p.stream_seed = w.embed.data_ptr(), w.stream_seed.data_ptr()
        p.collapse, p.final_norm = w.collapse.data_ptr(), w.final_norm.data_ptr()
        p.token, p.positions = self.token.data_ptr(), state.positions.data_ptr()
        for name in ("x", "proj", "normed", "scores", "stats", "mix", "partials", "hbuf", "ybuf",
                     "collapsed", "route_idx", "route_prob", "logits", "bar"):
            setattr(p, name, getattr(self, name).data_ptr())
        p.status = kernels.device_status(dev).data_ptr()
        p.head_part = self.head_part.data_ptr()
        self.params = p

    def prepare(self) -> None:
        """Fold the plain value rings a prefill left (v -> W_o v) unless this
        state already runs on folded rings."""
        st, c = self.state, self.model.cfg
        if getattr(st, "folded_rings", False):
            return
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("fold the CSA value rings (PersistentDecode.prepare) before "
                               "capturing the decode step in a CUDA graph")
        for j, b in enumerate(self.model.w.blocks):
            if not isinstance(b.mixer, CsaBlock):
                continue
            for i in range(c.num_loops):
                key = state_key(i, j)
                v = st.local_v[key]
                st.local_vo[key].copy_(
                    torch.matmul(v.view(-1, v.shape[-1]), b.mixer.w_o.t()).view_as(v))
        st.folded_rings = True

    def step(self, ids: torch.Tensor, out_token: torch.Tensor | None = None,
             logprob: torch.Tensor | None = None, seen: torch.Tensor | None = None,
             n_loops: int | None = None) -> torch.Tensor:
        """One decode token: ids [1] (device).  Returns the logits [1, V] fp32
        (this object's buffer, rewritten by the next step).  With out_token
        ([1] int64, may be `ids` itself) the step also samples greedily in the
        same launch: the first maximal logit's index, its raw log-softmax into
        logprob ([1] fp32) and its bit into seen ([ceil(V/32)] int32).
        n_loops: run the first n loops (default all), as the reference's
        model_step does for a smaller num_loops (model.cpp:1824-1825)."""
        nl = self.model.cfg.num_loops
        n_loops = nl if n_loops is None else int(n_loops)
        if not 1 <= n_loops <= nl:
            raise ValueError(f"n_loops must be in [1, {nl}], got {n_loops}")
        self.prepare()
        self.token.copy_(ids.reshape(-1)[:1])
        p = self.params
        p.n_loops = n_loops
        for name, t in (("out_token", out_token), ("out_logprob", logprob), ("seen", seen)):
            if t is not None and (not t.is_cuda or not t.is_contiguous()):
                raise ValueError(f"{name} must be a contiguous CUDA tensor")
        if out_token is not None and out_token.dtype != torch.int64:
            raise ValueError("out_token must be int64")
        p.out_token = 0 if out_token is None else out_token.data_ptr()
        p.out_logprob = 0 if logprob is None else logprob.data_ptr()
        p.seen = 0 if seen is None else seen.data_ptr()
        _native.call("llmyb_decode_persistent", C.byref(p), torch.cuda.current_stream().cuda_stream)
        return self.logits
