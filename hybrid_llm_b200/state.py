"""Device-resident recurrent state carried between tokens and loop passes.

Mirrors RecurrentState (model/recurrent_state.py:76-98): per loop pass and
block, keyed ``"loop{i}.core.{j}"`` exactly as PhysicalBlock builds its state
keys (model/model.py:168-171) —
  * ``gdn_states[key]``         [B, H, K, V] fp32 delta-rule state
  * ``gdn_conv_histories[key]`` [B, 3, D] bf16, last three GDN block inputs
  * ``local_k[key]`` / ``local_v[key]``  ring caches [B, W, H*Dh] / [B, W, D]
    of the CSA window (token p at slot p % W).  The reference keeps the
    normed hidden rows and re-projects K/V every step (csa.py:176-178); the
    cache holds the same projections computed once.
  * ``router_latents[key]``    [B, W, L] fp32 ring of the router's LayerNorm'd
    MLA latents of the last W positions (router_latent_histories,
    model/model.py:239-247; only with the router's local context).
  * CSA remote branch (only with ``csa_compression``): ``remote_k[key]``
    [B, C, H*Dh] / ``remote_v[key]`` [B, C, D] bf16, the keys and values of
    the row's completed block summaries (compressed memory keys / values,
    csa.py:208-256), ``remote_count[key]`` [B] int32 how many there are,
    ``remote_sum[key]`` [B, D] fp32 / ``remote_pending[key]`` [B] int32 the
    pending partial block (MemoryState.pending_sum / pending_count).  C =
    ceil(max_len / ratio) summaries.  The reference also appends an
    invisible entry for every decode token that completes no block; no query
    can see those, so they are not kept.
  * ``local_vo[key]`` [B, W, D] bf16: the CSA value ring folded with the
    block's output projection (W_o v), kept by the batch-1 persistent decode
    step (persistent.py) once ``folded_rings`` is set; the plain ``local_v``
    then falls behind until the next prefill.
  * ``positions`` [B] int32, position of the next token of each row.
All buffers are allocated once for a batch size so that a captured decode
graph can update them in place.
"""
from __future__ import annotations

import torch

from .config import HybridConfig


def state_key(loop: int, block: int) -> str:
    return f"loop{loop}.core.{block}"


class RecurrentState:
    def __init__(self, cfg: HybridConfig, batch: int, device: torch.device | str = "cuda",
                 max_len: int = 8192):
        """max_len: the longest sequence (prompt + generated tokens) the CSA
        remote branch's summary memory holds."""
        self.cfg = cfg
        self.batch = int(batch)
        self.max_len = int(max_len)
        self.device = torch.device(device)
        d = cfg.d_model
        self.gdn_states: dict[str, torch.Tensor] = {}
        self.gdn_conv_histories: dict[str, torch.Tensor] = {}
        self.local_k: dict[str, torch.Tensor] = {}
        self.local_v: dict[str, torch.Tensor] = {}
        for i in range(cfg.num_loops):
            for j in range(cfg.n_blocks):
                key = state_key(i, j)
                if cfg.block_kind(j) == "gdn":
                    self.gdn_states[key] = torch.zeros(
                        batch, cfg.gdn_heads, cfg.gdn_key_dim, cfg.gdn_value_dim,
                        dtype=torch.float32, device=self.device)
                    self.gdn_conv_histories[key] = torch.zeros(
                        batch, cfg.conv_kernel - 1, d, dtype=torch.bfloat16, device=self.device)
                else:
                    self.local_k[key] = torch.zeros(
                        batch, cfg.csa_window, cfg.csa_heads * cfg.csa_head_dim,
                        dtype=torch.bfloat16, device=self.device)
                    self.local_v[key] = torch.zeros(batch, cfg.csa_window, d,
                                                    dtype=torch.bfloat16, device=self.device)
        # router local context: the LayerNorm'd latents of the last W positions
        # (position p at slot p % W) per loop and block
        self.router_latents: dict[str, torch.Tensor] = {}
        if cfg.router_context:
            for i in range(cfg.num_loops):
                for j in range(cfg.n_blocks):
                    self.router_latents[state_key(i, j)] = torch.zeros(
                        batch, cfg.router_local_context, cfg.router_latent_dim,
                        dtype=torch.float32, device=self.device)
        self.remote_k: dict[str, torch.Tensor] = {}
        self.remote_v: dict[str, torch.Tensor] = {}
        self.remote_count: dict[str, torch.Tensor] = {}
        self.remote_sum: dict[str, torch.Tensor] = {}
        self.remote_pending: dict[str, torch.Tensor] = {}
        if cfg.csa_compression:
            cap = -(-self.max_len // cfg.csa_compression)
            hd = cfg.csa_heads * cfg.csa_head_dim
            for key in self.local_k:
                self.remote_k[key] = torch.zeros(batch, cap, hd, dtype=torch.bfloat16,
                                                 device=self.device)
                self.remote_v[key] = torch.zeros(batch, cap, d, dtype=torch.bfloat16,
                                                 device=self.device)
                self.remote_count[key] = torch.zeros(batch, dtype=torch.int32, device=self.device)
                self.remote_sum[key] = torch.zeros(batch, d, dtype=torch.float32,
                                                   device=self.device)
                self.remote_pending[key] = torch.zeros(batch, dtype=torch.int32,
                                                       device=self.device)
        self.local_vo: dict[str, torch.Tensor] = {}
        self.folded_rings = False
        self.positions = torch.zeros(batch, dtype=torch.int32, device=self.device)

    def _tables(self):
        return (("gdn_states", self.gdn_states), ("gdn_conv_histories", self.gdn_conv_histories),
                ("local_k", self.local_k), ("local_v", self.local_v),
                ("router_latents", self.router_latents), ("remote_k", self.remote_k),
                ("remote_v", self.remote_v), ("remote_count", self.remote_count),
                ("remote_sum", self.remote_sum), ("remote_pending", self.remote_pending),
                ("local_vo", self.local_vo))

    def fill_synthetic(self, position: int, seed: int = 0) -> None:
        """Stand-in for a prefilled context of `position` tokens (benchmarks
        whose cost does not depend on the context's values): ring caches and
        conv histories ~ N(0, 1), GDN states ~ N(0, 0.05), positions =
        position.  Drawn on the device from a seeded generator."""
        g = torch.Generator(device=self.device)
        g.manual_seed(int(seed))
        for t in (*self.local_k.values(), *self.local_v.values(),
                  *self.gdn_conv_histories.values()):
            t.copy_(torch.randn(t.shape, generator=g, device=self.device, dtype=torch.float32))
        for t in self.gdn_states.values():
            t.normal_(0.0, 0.05, generator=g)
        self.positions.fill_(int(position))

    def reset_rows(self, rows: torch.Tensor) -> None:
        """Clear the state of the selected rows (recurrent_state.py:218-244)."""
        mask = rows.to(device=self.device, dtype=torch.bool)
        for t in (*self.gdn_states.values(), *self.gdn_conv_histories.values(),
                  *self.router_latents.values(), *self.remote_count.values(),
                  *self.remote_sum.values(), *self.remote_pending.values()):
            t[mask] = 0
        self.positions[mask] = 0

    def zero_(self) -> None:
        """Zero every state tensor and position (a fresh conversation); on a
        CUDA device one native launch over a table of the tensors' regions,
        built on the first call (make that call before capturing it in a CUDA
        graph) and rebuilt when a table's tensors change."""
        tensors = [t for _, table in self._tables() for t in table.values()] + [self.positions]
        if self.device.type != "cuda":
            for t in tensors:
                t.zero_()
            return
        from . import kernels
        key = tuple((t.data_ptr(), t.numel() * t.element_size()) for t in tensors)
        if getattr(self, "_zero_key", None) != key:
            self._zero_table, self._zero_max = kernels.region_table(tensors, self.device)
            self._zero_key = key
        kernels.zero_regions(self._zero_table, self._zero_max)

    def nbytes(self) -> int:
        tensors = [t for _, table in self._tables() for t in table.values()] + [self.positions]
        return sum(t.numel() * t.element_size() for t in tensors)

    def state_dict(self) -> dict[str, torch.Tensor]:
        out: dict[str, torch.Tensor] = {"positions": self.positions.clone(),
                                        "folded_rings": torch.tensor(self.folded_rings)}
        for name, table in self._tables():
            for key, t in table.items():
                out[f"{name}.{key}"] = t.clone()
        return out

    def load_state_dict(self, sd: dict[str, torch.Tensor]) -> None:
        """Tables missing from `sd` (the folded rings of a state saved before
        the persistent step created them) keep their contents."""
        self.positions.copy_(sd["positions"])
        self.folded_rings = bool(sd.get("folded_rings", torch.tensor(False)))
        for name in sd:  # folded rings this state has not created yet
            key = name[len("local_vo."):]
            if name.startswith("local_vo.") and key not in self.local_vo:
                self.local_vo[key] = torch.empty_like(self.local_v[key])
        for name, table in self._tables():
            for key, t in table.items():
                if name == "local_vo" and f"{name}.{key}" not in sd:
                    continue
                t.copy_(sd[f"{name}.{key}"])
