"""Looped hybrid stack forward / decode (numpy oracle, float64).

Restates LoopedHybridMoEForCausalLM.forward and decode_step
(model/model.py:530-707, :787-915) and PhysicalBlock.forward / forward_step
(:162-376) for the configuration subset the B200 path serves (one plain
residual stream or multi-stream hyper-connections shared across loops, plain
router, no shared experts, CSA remote branch off, no stem/tail), over a state
dict with the reference's parameter names.
"""
from __future__ import annotations

import numpy as np


def _fp(x):
    """float32 inputs stay float32 (timed CPU baseline); everything else is float64."""
    x = np.asarray(x)
    return x if x.dtype == np.float32 else x.astype(np.float64)

from . import attention, gdn, mhc, routing


def rmsnorm(x, w, eps=1e-6):
    """norms.py:13-16."""
    x = _fp(x)
    r = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    return x * r * (1.0 if w is None else _fp(w))


def _layernorm(x, w, b, eps=1e-5):
    """nn.LayerNorm (default eps 1e-5) over the last dimension."""
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    return (x - mu) / np.sqrt(var + eps) * w + b


def _to_numpy(v, dtype):
    if hasattr(v, "detach"):  # a torch tensor; bf16 widens exactly to fp32 first
        v = v.detach().cpu()
        v = (v.float() if v.is_floating_point() else v).numpy()
    return np.asarray(v, dtype=dtype)


class _LazyParams:
    """name -> array converted on first access.  Routed-expert weights are
    cached only while the cache stays under `expert_cache_bytes` (the
    large model's experts are 40 GB in fp32): past it they are converted
    again on every access."""

    def __init__(self, sd, dtype, expert_cache_bytes: int):
        self._sd, self._dtype = sd, dtype
        self._cache: dict = {}
        self._expert_budget = expert_cache_bytes

    def __getitem__(self, name):
        got = self._cache.get(name)
        if got is not None:
            return got
        a = _to_numpy(self._sd[name], self._dtype)
        if ".moe.experts." not in name:
            self._cache[name] = a
        elif a.nbytes <= self._expert_budget:
            self._expert_budget -= a.nbytes
            self._cache[name] = a
        return a

    def __contains__(self, name):
        return name in self._sd


class _ExpertStack:
    """w[e] -> expert e's weight of one projection, fetched on use (only the
    routed experts of a call are read)."""

    def __init__(self, p, prefix: str, name: str):
        self._p, self._prefix, self._name = p, prefix, name

    def __getitem__(self, e):
        return self._p[f"{self._prefix}experts.{int(e)}.{self._name}_proj.weight"]


class OracleModel:
    def __init__(self, cfg, sd, dtype=np.float64, lazy: bool = False,
                 expert_cache_bytes: int = 0):
        """cfg: hybrid_llm_b200.config.HybridConfig-like; sd: name -> array-like.
        dtype float32 is used for the timed CPU baseline, float64 for parity.
        lazy: convert parameters on first use instead of all up front, and read
        only the routed experts' weights (for models too large to hold in host
        memory at `dtype`); expert_cache_bytes bounds the expert weights kept."""
        self.cfg = cfg
        self.dtype = dtype
        self.lazy = lazy
        if lazy:
            self.p = _LazyParams(sd, dtype, expert_cache_bytes)
        else:
            self.p = {k: _to_numpy(v, dtype) for k, v in sd.items()}
        self._experts: dict[int, tuple] = {}
        # Routing records / overrides, in call order (one entry per MoE call):
        # route_log collects (own top-k indices, own fp32 router logits);
        # forced_routes, when set, is a list of top-k index arrays that the
        # calls take instead of their own top-k (probabilities are still the
        # softmax of this model's own logits at those experts, context_router.py:73-74).
        self.route_log: list | None = None
        self.forced_routes: list | None = None

    def _gdn_params(self, j):
        p = f"recurrent_core.{j}.mixer."
        g = lambda n: self.p[p + n]
        return dict(q_proj=g("q_proj.weight"), k_proj=g("k_proj.weight"), v_proj=g("v_proj.weight"),
                    beta_proj=g("beta_proj.weight"), beta_bias=g("beta_proj.bias"),
                    gate_proj=g("gate_proj.weight"), out_proj=g("out_proj.weight"),
                    conv=g("conv.weight"), decay_logit=g("decay_logit"))

    def _csa_params(self, j):
        p = f"recurrent_core.{j}.mixer."
        names = ("query", "key", "value", "local_out", "out")
        if self.cfg.csa_compression:
            names += ("remote_out", "compressor.key", "compressor.value")
        return {n: self.p[p + n + ".weight"] for n in names}

    def _router_logits(self, j, m, state, key, step):
        """ContextAwareRouter.forward / forward_step (context_router.py:59-74,
        :89-133) without HCA latents, on m [B, T, D]: local = RMSNorm(m);
        with the local context, route_input = local + sigmoid(route_gate) *
        context_out(local_context_out(window mean of LayerNorm(down(local))))
        (mla_memory.py:23-48), the window being the last W tokens in prefill
        and the kept latent history plus the new token in a decode step."""
        c, p = self.cfg, f"recurrent_core.{j}.moe.router."
        g = lambda n: self.p[p + n]
        local = rmsnorm(m, g("norm.weight"), c.rms_eps)
        if not c.router_context:
            return local @ g("logits.weight").T
        z = local @ g("latent_memory.down.weight").T
        mu = z.mean(-1, keepdims=True)
        var = ((z - mu) ** 2).mean(-1, keepdims=True)
        lat = (z - mu) / np.sqrt(var + 1e-5) * g("latent_memory.norm.weight") + \
            g("latent_memory.norm.bias")
        w = c.router_local_context
        if step:
            hist = np.concatenate([state["rlat"][key], lat], axis=1)[:, -w:]
            state["rlat"][key] = hist
            box = hist.mean(1, keepdims=True)
        else:
            box = np.stack([lat[:, max(0, t - w + 1):t + 1].mean(1) for t in range(lat.shape[1])], 1)
            state["rlat"][key] = lat[:, -w:]
        ctx = (box @ g("local_context_out.weight").T) @ g("context_out.weight").T
        gate = 1.0 / (1.0 + np.exp(-np.asarray(g("route_gate"), dtype=np.float64)))
        return (local + gate * ctx) @ g("logits.weight").T

    def _moe(self, j, m, state=None, key=None, step=False):
        """SparseMoE.forward (moe.py:172-199) without shared experts."""
        c, p = self.cfg, f"recurrent_core.{j}.moe."
        lead = m.shape[:-1]
        flat = m.reshape(-1, m.shape[-1])
        logits = self._router_logits(j, m, state, key, step).reshape(flat.shape[0], -1)
        idx, prob = routing.router_topk(logits.astype(np.float32), c.moe_top_k)
        if self.route_log is not None:
            self.route_log.append((idx, logits.astype(np.float32)))
        if self.forced_routes is not None:
            idx = np.asarray(self.forced_routes.pop(0), dtype=np.int64).reshape(idx.shape)
            top = np.take_along_axis(logits.astype(np.float32).astype(np.float64), idx, -1)
            prob = np.exp(top - top.max(-1, keepdims=True))
            prob = prob / prob.sum(-1, keepdims=True)
        if j not in self._experts:
            e = c.moe_experts
            if self.lazy:
                self._experts[j] = tuple(_ExpertStack(self.p, p, n) for n in ("gate", "up", "down"))
            else:
                self._experts[j] = tuple(
                    np.stack([self.p[f"{p}experts.{x}.{n}_proj.weight"] for x in range(e)])
                    for n in ("gate", "up", "down"))
        wg, wu, wd = self._experts[j]
        out = routing.moe_forward(flat, idx, prob, wg, wu, wd, dtype=self.dtype)
        if c.moe_shared:
            # shared experts (moe.py:185-198): every token, sum / sqrt(n_shared)
            x = np.asarray(flat, dtype=out.dtype)
            for s in range(c.moe_shared):
                q = f"{p}shared.{s}."
                g_ = x @ self.p[q + "gate_proj.weight"].T
                u_ = x @ self.p[q + "up_proj.weight"].T
                out = out + ((routing.silu(g_) * u_) @ self.p[q + "down_proj.weight"].T
                             ) / np.sqrt(c.moe_shared)
        return out.reshape(*lead, -1), logits

    def _read(self, j, x, norm):
        """Sub-layer input (PhysicalBlock._read + its RMSNorm, model.py:119-123):
        returns (normed, maps); maps is None on the plain residual stream."""
        c, w = self.cfg, self.p[f"recurrent_core.{j}.{norm}.weight"]
        if not c.mhc_streams:
            return rmsnorm(x, w, c.rms_eps), None
        maps, hidden = mhc.read(x, self.p, f"recurrent_core.{j}.mhc.", c.mhc_streams,
                                c.mhc_iterations)
        return rmsnorm(hidden, w, c.rms_eps), maps

    # -------------------------------------------------------- loop memory
    def _streams_mean(self, x):
        """The token's hidden state as the hook sees it: the mean over the
        streams (loop_memory.py:38, :45); x itself on one plain stream."""
        return x.mean(-2) if self.cfg.mhc_streams else x

    def _lm_encode(self, x):
        """LoopMemoryHook.encode / record (loop_memory.py:36-38, :54-66):
        LayerNorm(down(mean over streams)), the endpoint of one loop."""
        p = "loop_memory.compressor."
        h = self._streams_mean(x) @ self.p[p + "down.weight"].T
        return _layernorm(h, self.p[p + "norm.weight"], self.p[p + "norm.bias"])

    def _lm_inject(self, x, endpoints):
        """LoopMemoryHook.inject (loop_memory.py:40-52) with LatentAttention
        (mla_memory.py:66-86, causal=False, no key mask): every token attends
        over its own endpoints of the earlier loops; the gated output is added
        to every stream."""
        if not endpoints:
            return x
        c, p = self.cfg, "loop_memory."
        h, hd = c.loop_memory_heads, c.loop_memory_head_dim
        qn = _layernorm(self._streams_mean(x), self.p[p + "query_norm.weight"],
                        self.p[p + "query_norm.bias"])
        lead = qn.shape[:-1]
        q = (qn @ self.p[p + "attention.q.weight"].T).reshape(*lead, h, hd)
        mem = np.stack(endpoints, axis=-2)                      # [..., J, L]
        k = (mem @ self.p[p + "attention.k.weight"].T).reshape(*lead, len(endpoints), h, hd)
        v = (mem @ self.p[p + "attention.v.weight"].T).reshape(*lead, len(endpoints), h, hd)
        s = np.einsum("...hd,...jhd->...hj", q, k) / np.sqrt(hd)
        s = np.exp(s - s.max(-1, keepdims=True))
        prob = s / s.sum(-1, keepdims=True)
        o = np.einsum("...hj,...jhd->...hd", prob, v).reshape(*lead, h * hd)
        o = o @ self.p[p + "attention.o.weight"].T
        gate = 1.0 / (1.0 + np.exp(-np.asarray(self.p[p + "gating_logit"], dtype=np.float64)))
        gate = np.asarray(gate, dtype=o.dtype)
        return x + gate * (o[..., None, :] if c.mhc_streams else o)

    def _write(self, j, x, update, maps):
        """PhysicalBlock._write (model.py:125-126)."""
        if maps is None:
            return x + update
        return mhc.write(x, update, maps, self.p, f"recurrent_core.{j}.mhc.")

    def new_state(self, batch):
        c = self.cfg
        st = {"gdn": {}, "conv": {}, "hist": {}, "rlat": {}, "cmem": {},
              "pos": np.zeros(batch, dtype=np.int64)}
        for i in range(c.num_loops):
            for j in range(c.n_blocks):
                if c.block_kind(j) == "gdn":
                    st["gdn"][(i, j)] = np.zeros((batch, c.gdn_heads, c.gdn_key_dim, c.gdn_value_dim),
                                                 dtype=self.dtype)
        return st

    def run_stack(self, streams, state, loops=None, router_logits=None):
        """Recurrent core over streams [B,T,D] (model/model.py:618-687)."""
        c = self.cfg
        loops = c.num_loops if loops is None else loops
        x = _fp(streams)
        t = x.shape[1]
        endpoints = []  # loop memory (model/model.py:608, :636, :661-667)
        for i in range(loops):
            if c.loop_memory:
                x = self._lm_inject(x, endpoints)
            for j in range(c.n_blocks):
                normed, maps = self._read(j, x, "mixer_norm")
                if c.block_kind(j) == "gdn":
                    mixed, s = gdn.gdn_layer(normed, self._gdn_params(j), state["gdn"][(i, j)])
                    state["gdn"][(i, j)] = s
                    state["conv"][(i, j)] = normed[:, -(c.conv_kernel - 1):]
                elif c.csa_compression:
                    mixed, state["cmem"][(i, j)] = attention.csa_layer_remote(
                        normed, self._csa_params(j), c.csa_heads, c.csa_window, c.csa_compression,
                        c.csa_top_k)
                    state["hist"][(i, j)] = normed[:, -(c.csa_window - 1):]
                else:
                    mixed = attention.csa_layer(normed, self._csa_params(j), c.csa_heads, c.csa_window)
                    state["hist"][(i, j)] = normed[:, -(c.csa_window - 1):]
                x = self._write(j, x, mixed, maps)
                m, maps = self._read(j, x, "ffn_norm")
                y, lg = self._moe(j, m, state, (i, j))
                if router_logits is not None:
                    router_logits.append(lg)
                x = self._write(j, x, y, maps)
            if c.loop_memory:
                endpoints.append(self._lm_encode(x))
        state["pos"][:] = t
        return x

    def head(self, x):
        c = self.cfg
        x = np.asarray(x)
        if c.mhc_streams:
            x = x.reshape(*x.shape[:-2], -1)
        col = x @ self.p["mhc_collapse.weight"].T
        h = rmsnorm(col, self.p["final_norm.weight"], c.rms_eps)
        return h @ self.p["embed_tokens.weight"].T

    def embed(self, ids):
        e = self.p["embed_tokens.weight"][np.asarray(ids)]
        if self.cfg.mhc_streams:
            return e[..., None, :] + self.p["stream_seed"].reshape(self.cfg.mhc_streams, -1)
        return e + self.p["stream_seed"].reshape(-1)

    def forward(self, ids, state=None):
        ids = np.asarray(ids)
        state = self.new_state(ids.shape[0]) if state is None else state
        x = self.run_stack(self.embed(ids), state)
        return self.head(x), state

    def decode_step(self, ids, state):
        """model/model.py:787-915 with PhysicalBlock.forward_step (:266-376)."""
        c = self.cfg
        ids = np.asarray(ids).reshape(-1)
        x = self.embed(ids)[:, None, :]
        endpoints = []  # loop memory of this step (model/model.py:840, :877, :884-891)
        for i in range(c.num_loops):
            if c.loop_memory:
                x = self._lm_inject(x, endpoints)
            for j in range(c.n_blocks):
                normed, maps = self._read(j, x, "mixer_norm")
                if c.block_kind(j) == "gdn":
                    hist = state["conv"][(i, j)]
                    if hist.shape[1] < c.conv_kernel - 1:
                        pad = np.zeros((hist.shape[0], c.conv_kernel - 1 - hist.shape[1], hist.shape[2]),
                                       dtype=hist.dtype)
                        hist = np.concatenate([pad, hist], axis=1)
                    mixed, s = gdn.gdn_layer(normed, self._gdn_params(j), state["gdn"][(i, j)],
                                             conv_history=hist)
                    state["gdn"][(i, j)] = s
                    state["conv"][(i, j)] = np.concatenate([hist, normed], axis=1)[:, 1:]
                else:
                    a = self._csa_params(j)
                    win = np.concatenate([state["hist"][(i, j)], normed], axis=1)[:, -c.csa_window:]
                    b_, L, _ = win.shape
                    q = (normed[:, 0] @ a["query"].T).reshape(b_, c.csa_heads, -1)
                    k = (win @ a["key"].T).reshape(b_, L, c.csa_heads, -1)
                    v = win @ a["value"].T
                    local = attention.csa_local_step(q, k, v)
                    out = local @ a["local_out"].T
                    if c.csa_compression:
                        pos = int(state["pos"][0])
                        mem = attention.compress_step(state["cmem"][(i, j)], normed[:, 0],
                                                      a["compressor.key"], a["compressor.value"],
                                                      c.csa_compression, pos)
                        remote = attention.remote_attention(q[:, None], mem["keys"], mem["values"],
                                                            mem["pos"], np.array([pos]), c.csa_top_k)
                        out = out + remote[:, 0] @ a["remote_out"].T
                    mixed = (out @ a["out"].T)[:, None, :]
                    state["hist"][(i, j)] = win[:, -(c.csa_window - 1):]
                x = self._write(j, x, mixed, maps)
                m, maps = self._read(j, x, "ffn_norm")
                y, _ = self._moe(j, m, state, (i, j), step=True)
                x = self._write(j, x, y, maps)
            if c.loop_memory:
                endpoints.append(self._lm_encode(x))
        state["pos"] += 1
        return self.head(x[:, 0]), state
