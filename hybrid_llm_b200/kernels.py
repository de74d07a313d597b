"""Torch-tensor wrappers around the llmyb C ABI.

Each wrapper validates dtypes/contiguity on the host, allocates outputs and
scratch with torch's caching allocator (the kernels themselves never
allocate) and launches on torch's current CUDA stream.  Nothing here has a
CPU path: tensors must live on a CUDA device.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _native

TILE_M = 256  # rows per grouped-GEMM tile (a CTA pair); the plan's tile_offsets use it

_status: dict[int, torch.Tensor] = {}


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _require_cuda(*tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("llmyb kernels take CUDA tensors only (no CPU fallback)")


def _inplace(t: torch.Tensor, name: str) -> torch.Tensor:
    """Tensors a kernel writes in place must already be dense."""
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous (it is updated in place)")
    return t


def _rows(t: torch.Tensor, name: str) -> None:
    """[rows, cols] views read with a row stride need a unit column stride."""
    if t.stride(-1) != 1:
        raise ValueError(f"{name}: the last dimension must be contiguous")


def device_status(device: torch.device | None = None) -> torch.Tensor:
    """Per-device int32 word the kernels set when a bounded wait gives up."""
    idx = torch.cuda.current_device() if device is None else torch.device(device).index or 0
    buf = _status.get(idx)
    if buf is None:
        buf = torch.zeros(1, dtype=torch.int32, device=f"cuda:{idx}")
        _status[idx] = buf
    return buf


def check_device_status(device: torch.device | None = None) -> None:
    """Synchronize and raise if any kernel recorded a device-side error."""
    buf = device_status(device)
    code = int(buf.item())
    if code != 0:
        buf.zero_()
        _native.check(code, "device-side status")


def launch_count() -> int:
    """Kernel launches issued by the native library so far (host-side count)."""
    return int(_native.lib().llmyb_launch_count())


@dataclass
class RoutePlan:
    """Top-k routes and the expert-grouped dispatch order (all on device)."""

    topk_idx: torch.Tensor      # [N, k] int64
    topk_prob: torch.Tensor     # [N, k] fp32
    counts: torch.Tensor        # [E] int32
    offsets: torch.Tensor       # [E+1] int32, expert row ranges in permuted order
    tile_offsets: torch.Tensor  # [E+1] int32, 128-row tiles per expert (prefix)
    perm_token: torch.Tensor    # [N*k] int32, token of each permuted row
    perm_prob: torch.Tensor     # [N*k] fp32, route probability of each permuted row
    route_pos: torch.Tensor     # [N*k] int32, permuted row of route t*k+s
    sort_order: torch.Tensor | None  # [N*k] int64, flat route id of each permuted row
    tile_m: int = TILE_M             # rows per tile behind tile_offsets

    @property
    def n_experts(self) -> int:
        return self.counts.numel()


def _plan_buffers(n: int, e: int, k: int, device, with_sort_order: bool):
    i32 = dict(dtype=torch.int32, device=device)
    return dict(
        counts=torch.empty(e, **i32), offsets=torch.empty(e + 1, **i32),
        tile_offsets=torch.empty(e + 1, **i32), perm_token=torch.empty(n * k, **i32),
        perm_prob=torch.empty(n * k, dtype=torch.float32, device=device),
        route_pos=torch.empty(n * k, **i32),
        sort_order=torch.empty(n * k, dtype=torch.int64, device=device) if with_sort_order else None,
    )


def _plan_scratch(n: int, e: int, device) -> torch.Tensor:
    nbytes = int(_native.lib().llmyb_moe_plan_scratch_bytes(n, e))
    return torch.empty(max(nbytes, 4), dtype=torch.uint8, device=device)


def route(logits: torch.Tensor, k: int, bias: torch.Tensor | None = None, *,
          with_sort_order: bool = False, tile_m: int = TILE_M) -> RoutePlan:
    """Top-k + softmax + dispatch plan from fp32 router logits [N, E]."""
    _require_cuda(logits, bias)
    if logits.dtype != torch.float32 or logits.dim() != 2:
        raise ValueError("route expects fp32 logits of shape [N, E]")
    logits = logits.contiguous()
    n, e = logits.shape
    if bias is not None:
        bias = bias.to(torch.float32).contiguous()
    dev = logits.device
    idx = torch.empty(n, k, dtype=torch.int64, device=dev)
    prob = torch.empty(n, k, dtype=torch.float32, device=dev)
    b = _plan_buffers(n, e, k, dev, with_sort_order)
    scratch = _plan_scratch(n, e, dev)
    _native.call("llmyb_route", _ptr(logits), _ptr(bias), n, e, k, tile_m, _ptr(idx), _ptr(prob),
                 _ptr(b["counts"]), _ptr(b["offsets"]), _ptr(b["tile_offsets"]),
                 _ptr(b["perm_token"]), _ptr(b["perm_prob"]), _ptr(b["route_pos"]),
                 _ptr(b["sort_order"]), _ptr(scratch), _stream())
    return RoutePlan(idx, prob, **b, tile_m=tile_m)


def route_norm(m: torch.Tensor, router_norm: torch.Tensor, w_router: torch.Tensor, k: int,
               eps: float, bias: torch.Tensor | None = None, *, tile_m: int = TILE_M,
               logits_out: torch.Tensor | None = None,
               with_sort_order: bool = False) -> RoutePlan:
    """Prefill router (context_router.py:62-65 without the local context) from
    the FFN-normalised rows m [N, D] fp32: RMSNorm(m) * router_norm, fp32
    logits w_router [E, D] . r (into logits_out [N, E] if given), top-k +
    softmax and the dispatch plan."""
    _require_cuda(m, router_norm, w_router, bias, logits_out)
    if m.dtype != torch.float32 or w_router.dtype != torch.float32:
        raise ValueError("route_norm takes fp32 rows and router weights")
    m = m.contiguous()
    n, d = m.shape
    e = w_router.shape[0]
    if bias is not None:
        bias = bias.to(torch.float32).contiguous()
    if logits_out is not None:
        _inplace(logits_out, "logits_out")
    dev = m.device
    idx = torch.empty(n, k, dtype=torch.int64, device=dev)
    prob = torch.empty(n, k, dtype=torch.float32, device=dev)
    b = _plan_buffers(n, e, k, dev, with_sort_order)
    scratch = _plan_scratch(n, e, dev) if n * k > 2048 else None
    _native.call("llmyb_route_norm", _ptr(m), n, d, _ptr(router_norm.contiguous()),
                 _ptr(w_router.contiguous()), float(eps), _ptr(bias), e, k, tile_m,
                 _ptr(logits_out), _ptr(idx), _ptr(prob), _ptr(b["counts"]), _ptr(b["offsets"]),
                 _ptr(b["tile_offsets"]), _ptr(b["perm_token"]), _ptr(b["perm_prob"]),
                 _ptr(b["route_pos"]), _ptr(b["sort_order"]), _ptr(scratch), _stream())
    return RoutePlan(idx, prob, **b, tile_m=tile_m)


def route_norm_supported(d_model: int, n_experts: int) -> bool:
    return d_model % 4 == 0 and d_model <= 1024 and n_experts <= 256


def grouped_tile_m(n_rows: int, n_experts: int) -> int:
    """Rows per grouped-GEMM tile for a plan of n_rows routes: CTA-pair 256-row
    tiles once the average expert fills one, else single-CTA 128-row tiles
    (half the padding rows at a few dozen rows per expert)."""
    return TILE_M if n_rows >= TILE_M * n_experts else 128


def router_topk(logits: torch.Tensor, k: int, bias: torch.Tensor | None = None):
    """(indices int64, probabilities fp32) — context_router.py:73-74 semantics."""
    _require_cuda(logits, bias)
    logits = logits.to(torch.float32).contiguous()
    n, e = logits.shape
    idx = torch.empty(n, k, dtype=torch.int64, device=logits.device)
    prob = torch.empty(n, k, dtype=torch.float32, device=logits.device)
    _native.call("llmyb_router_topk", _ptr(logits), _ptr(bias), n, e, k, _ptr(idx), _ptr(prob),
                 _stream())
    return idx, prob


def moe_plan(topk_idx: torch.Tensor, topk_prob: torch.Tensor, n_experts: int, *,
             with_sort_order: bool = False, tile_m: int = TILE_M) -> RoutePlan:
    """Dispatch plan for externally computed top-k routes (moe.py:42-60)."""
    _require_cuda(topk_idx, topk_prob)
    idx = topk_idx.to(torch.int64).contiguous()
    prob = topk_prob.to(torch.float32).contiguous()
    n, k = idx.shape
    dev = idx.device
    b = _plan_buffers(n, n_experts, k, dev, with_sort_order)
    scratch = _plan_scratch(n, n_experts, dev)
    _native.call("llmyb_moe_plan", _ptr(idx), _ptr(prob), n, n_experts, k, tile_m,
                 _ptr(b["counts"]), _ptr(b["offsets"]), _ptr(b["tile_offsets"]),
                 _ptr(b["perm_token"]), _ptr(b["perm_prob"]), _ptr(b["route_pos"]),
                 _ptr(b["sort_order"]), _ptr(scratch), _ptr(device_status(dev)), _stream())
    return RoutePlan(idx, prob, **b, tile_m=tile_m)


def route_fused(streams: torch.Tensor, delta: torch.Tensor | None, ffn_norm: torch.Tensor,
                router_norm: torch.Tensor, w_router: torch.Tensor, k: int, eps: float,
                m_bf: torch.Tensor, tile_m: int = TILE_M, variant: str = "auto") -> RoutePlan:
    """Decode router: streams += delta; m_bf = RMSNorm_ffn(streams); top-k over
    w_router . RMSNorm_router(m) (fp32) and the dispatch plan.  variant
    "single": one CTA, one launch (N*E <= 256); "multi": route_decode (three
    launches, any N <= 256); "auto": single for N <= 4 and N*E <= 64.  Both
    variants give bit-identical results."""
    _require_cuda(streams, delta, ffn_norm, router_norm, w_router, m_bf)
    _inplace(streams, "streams")
    _inplace(m_bf, "m_bf")
    n, d = streams.shape
    e = w_router.shape[0]
    dev = streams.device
    idx = torch.empty(n, k, dtype=torch.int64, device=dev)
    prob = torch.empty(n, k, dtype=torch.float32, device=dev)
    b = _plan_buffers(n, e, k, dev, False)
    delta = None if delta is None else delta.contiguous()
    if variant == "multi" or (variant == "auto" and (n * e > 64 or n > 4)):
        # the single CTA normalises its tokens one after another and runs
        # 8 logit warps: worth one launch only for a few (token, expert) pairs
        return route_decode(streams, delta, ffn_norm, router_norm, w_router, k, eps, m_bf,
                            tile_m=tile_m)
    _native.call("llmyb_route_fused", _ptr(streams), _ptr(delta), n, d, _ptr(ffn_norm),
                 _ptr(router_norm), _ptr(w_router), float(eps), e, k, int(tile_m), _ptr(m_bf),
                 _ptr(idx), _ptr(prob), _ptr(b["counts"]), _ptr(b["offsets"]),
                 _ptr(b["tile_offsets"]), _ptr(b["perm_token"]), _ptr(b["perm_prob"]),
                 _ptr(b["route_pos"]), _stream())
    return RoutePlan(idx, prob, **b, tile_m=tile_m)


def route_decode(streams: torch.Tensor, delta: torch.Tensor | None, ffn_norm: torch.Tensor,
                 router_norm: torch.Tensor, w_router: torch.Tensor, k: int, eps: float,
                 m_bf: torch.Tensor, tile_m: int = TILE_M) -> RoutePlan:
    """route_fused with one CTA per token for the logits (any N <= 256), then
    one top-k/plan launch; bit-identical to the single-CTA route_fused."""
    _require_cuda(streams, delta, ffn_norm, router_norm, w_router, m_bf)
    _inplace(streams, "streams")
    _inplace(m_bf, "m_bf")
    n, d = streams.shape
    e = w_router.shape[0]
    dev = streams.device
    idx = torch.empty(n, k, dtype=torch.int64, device=dev)
    prob = torch.empty(n, k, dtype=torch.float32, device=dev)
    b = _plan_buffers(n, e, k, dev, False)
    delta = None if delta is None else delta.contiguous()
    logits = torch.empty(n * (d + e), dtype=torch.float32, device=dev)
    _native.call("llmyb_route_decode", _ptr(streams), _ptr(delta), n, d, _ptr(ffn_norm),
                 _ptr(router_norm), _ptr(w_router), float(eps), e, k, int(tile_m), _ptr(m_bf),
                 _ptr(logits), _ptr(idx), _ptr(prob), _ptr(b["counts"]), _ptr(b["offsets"]),
                 _ptr(b["tile_offsets"]), _ptr(b["perm_token"]), _ptr(b["perm_prob"]),
                 _ptr(b["route_pos"]), _stream())
    return RoutePlan(idx, prob, **b, tile_m=tile_m)


def route_fused_supported(n: int, e: int, k: int, d: int) -> bool:
    return n <= 256 and n * k <= 2048 and d % 4 == 0 and d <= 8192 and e <= 256 and k <= 32


def moe_decode_experts(x: torch.Tensor, plan: RoutePlan, w13: torch.Tensor, w2: torch.Tensor,
                       y_rows: torch.Tensor | None = None,
                       h_scratch: torch.Tensor | None = None) -> torch.Tensor:
    """Routed expert outputs p * expert(x) per route in plan order ([N*k, D] bf16),
    to be combined by add_rmsnorm_routed."""
    _require_cuda(x, w13, w2)
    x = x.contiguous()
    n, d = x.shape
    k = plan.topk_idx.shape[1]
    e, f2, _ = w13.shape
    f = f2 // 2
    if y_rows is None:
        y_rows = torch.empty(n * k, d, dtype=torch.bfloat16, device=x.device)
    if h_scratch is None:
        h_scratch = torch.empty(n * k, f, dtype=torch.bfloat16, device=x.device)
    _native.call("llmyb_moe_decode_experts", _ptr(x), n, d, k, _ptr(plan.perm_token),
                 _ptr(plan.perm_prob), _ptr(plan.offsets), e, _ptr(w13), _ptr(w2), f,
                 _ptr(h_scratch), _ptr(y_rows), _stream())
    return y_rows


def moe_decode_experts_to(x: torch.Tensor, n_rows: int, perm_token: torch.Tensor,
                          perm_prob: torch.Tensor, offsets: torch.Tensor, w13: torch.Tensor,
                          w2: torch.Tensor, h_scratch: torch.Tensor, y_out: torch.Tensor,
                          out_row: torch.Tensor) -> None:
    """y_out[out_row[pos]] = p * expert(x[perm_token[pos]]) over an explicit plan
    of at most n_rows positions (offsets [E+1] on the device)."""
    _require_cuda(x, perm_token, perm_prob, offsets, w13, w2, h_scratch, y_out, out_row)
    _inplace(y_out, "y_out")
    _inplace(h_scratch, "h_scratch")
    e, f2, d = w13.shape
    if x.shape[-1] != d or h_scratch.numel() < n_rows * (f2 // 2):
        raise ValueError("moe_decode_experts_to: shape mismatch")
    _native.call("llmyb_moe_decode_experts_to", _ptr(x), int(n_rows), d, _ptr(perm_token),
                 _ptr(perm_prob), _ptr(offsets), e, _ptr(w13), _ptr(w2), f2 // 2,
                 _ptr(h_scratch), _ptr(y_out), _ptr(out_row), _stream())


def ep_header_rows(experts_per_rank: int, capacity: int, d_model: int) -> int:
    """Header rows of an expert-parallel dispatch segment."""
    h = int(_native.lib().llmyb_ep_header_rows(experts_per_rank, capacity, d_model))
    if h < 0:
        raise ValueError("ep_header_rows: invalid arguments")
    return h


def ep_dispatch_pack(x: torch.Tensor, plan: RoutePlan, n_experts: int, world: int,
                     capacity: int, send: torch.Tensor, ret_route_pos: torch.Tensor) -> None:
    """Pack the W dispatch segments (send [W*(H+C), D]) from a local plan and
    write the return-buffer row of every route into ret_route_pos."""
    _require_cuda(x, send, ret_route_pos)
    x = x.contiguous()
    _inplace(send, "send")
    _inplace(ret_route_pos, "ret_route_pos")
    n_routes = plan.perm_token.numel()
    if ret_route_pos.numel() < n_routes:
        raise ValueError("ret_route_pos too small")
    _native.call("llmyb_ep_dispatch_pack", _ptr(x), x.shape[-1], _ptr(plan.offsets),
                 _ptr(plan.perm_token), _ptr(plan.perm_prob), _ptr(plan.route_pos), n_routes,
                 int(n_experts), int(world), int(capacity), _ptr(send), _ptr(ret_route_pos),
                 _stream())


def ep_recv_plan(recv: torch.Tensor, world: int, capacity: int, experts_per_rank: int,
                 offsets_l: torch.Tensor, perm_token_l: torch.Tensor, perm_prob_l: torch.Tensor,
                 out_row: torch.Tensor, tile_offsets_l: torch.Tensor | None = None,
                 tile_m: int = 128, wait_flags: torch.Tensor | None = None,
                 sync: torch.Tensor | None = None) -> None:
    """Expert-ordered plan over the received dispatch segments (after a bounded
    wait for the peers' dispatch flags when wait_flags is given)."""
    _require_cuda(recv, offsets_l, perm_token_l, perm_prob_l, out_row, tile_offsets_l, wait_flags,
                  sync)
    for t, n in ((offsets_l, "offsets_l"), (perm_token_l, "perm_token_l"),
                 (perm_prob_l, "perm_prob_l"), (out_row, "out_row")):
        _inplace(t, n)
    status = device_status(recv.device) if wait_flags is not None else None
    _native.call("llmyb_ep_recv_plan", _ptr(recv), recv.shape[-1], int(world), int(capacity),
                 int(experts_per_rank), int(tile_m), _ptr(offsets_l), _ptr(tile_offsets_l),
                 _ptr(perm_token_l), _ptr(perm_prob_l), _ptr(out_row), _ptr(wait_flags),
                 _ptr(sync), _ptr(status), _stream())


def ep_dispatch_p2p(x: torch.Tensor, plan: RoutePlan, n_experts: int, world: int, capacity: int,
                    peer_segs: int, peer_flags: int, sync: torch.Tensor,
                    ret_route_pos: torch.Tensor) -> None:
    """Dispatch segments stored straight into the peers' receive buffers.
    peer_segs / peer_flags: host addresses of arrays of W device pointers."""
    _require_cuda(x, sync, ret_route_pos)
    x = x.contiguous()
    n_routes = plan.perm_token.numel()
    _native.call("llmyb_ep_dispatch_p2p", _ptr(x), x.shape[-1], _ptr(plan.offsets),
                 _ptr(plan.perm_token), _ptr(plan.perm_prob), _ptr(plan.route_pos), n_routes,
                 int(n_experts), int(world), int(capacity), peer_segs, peer_flags, _ptr(sync),
                 _ptr(ret_route_pos), _stream())


def ep_return_p2p(ret_send: torch.Tensor, recv: torch.Tensor, world: int, capacity: int,
                  experts_per_rank: int, peer_segs: int, peer_flags: int,
                  sync: torch.Tensor) -> None:
    """Expert outputs pushed back into the source ranks' return buffers."""
    _require_cuda(ret_send, recv, sync)
    _native.call("llmyb_ep_return_p2p", _ptr(ret_send), _ptr(recv), ret_send.shape[-1], int(world),
                 int(capacity), int(experts_per_rank), peer_segs, peer_flags, _ptr(sync), _stream())


def ep_wait(flags: torch.Tensor, world: int, sync: torch.Tensor, limit_ns: int = 0) -> None:
    """Bounded device-side wait for the current exchange round's flags; after
    limit_ns (0: one second) the device status word gets LLMYB_ETIMEOUT."""
    _require_cuda(flags, sync)
    _native.call("llmyb_ep_wait", _ptr(flags), int(world), _ptr(sync),
                 _ptr(device_status(flags.device)), int(limit_ns), _stream())


def grouped_scratch_bytes(n_rows: int, d_model: int, ffn: int) -> int:
    """Scratch of moe_grouped_experts_to for a plan of n_rows positions."""
    return int(_native.lib().llmyb_moe_grouped_scratch_bytes(int(n_rows), 1, int(d_model), int(ffn)))


def grouped_shape_ok(d_model: int, ffn: int) -> bool:
    """Shapes the tcgen05 grouped GEMMs tile: 256-column output tiles of both
    products (d_model % 256, 2 * ffn % 256) and 64-wide K blocks."""
    return d_model % 256 == 0 and ffn % 128 == 0


def use_grouped_rows(n_rows: int, n_experts: int, d_model: int | None = None,
                     ffn: int | None = None) -> bool:
    """Routed rows per expert at which the tcgen05 grouped GEMMs beat the
    weight-streaming decode kernels (whose CUDA-core work grows with rows),
    for shapes the grouped GEMMs support."""
    if d_model is not None and ffn is not None and not grouped_shape_ok(d_model, ffn):
        return False
    return n_rows >= 2 * n_experts


def moe_grouped_experts_to(x: torch.Tensor, n_rows: int, perm_token: torch.Tensor,
                           perm_prob: torch.Tensor, offsets: torch.Tensor,
                           tile_offsets: torch.Tensor, tile_m: int, w13: torch.Tensor,
                           w2: torch.Tensor, scratch: torch.Tensor, y_out: torch.Tensor,
                           out_row: torch.Tensor | None = None) -> None:
    """y_out[out_row[pos] or pos] = p * expert(x[perm_token[pos]]) on the tcgen05
    grouped GEMMs, pos < offsets[E] (read on the device)."""
    _require_cuda(x, perm_token, perm_prob, offsets, tile_offsets, w13, w2, scratch, y_out, out_row)
    _inplace(y_out, "y_out")
    x = x.contiguous()
    e, f2, d = w13.shape
    if scratch.numel() < grouped_scratch_bytes(n_rows, d, f2 // 2):
        raise ValueError("moe_grouped_experts_to: scratch too small")
    _native.call("llmyb_moe_grouped_experts_to", _ptr(x), d, int(n_rows), _ptr(perm_token),
                 _ptr(perm_prob), _ptr(offsets), _ptr(tile_offsets), int(tile_m), e, _ptr(w13),
                 _ptr(w2), f2 // 2, _ptr(scratch), _ptr(y_out), _ptr(out_row),
                 _ptr(device_status(x.device)), _stream())


def moe_experts_rows(x: torch.Tensor, plan: RoutePlan, w13: torch.Tensor, w2: torch.Tensor,
                     y_rows: torch.Tensor | None = None, path: str = "auto") -> torch.Tensor:
    """Routed expert outputs p * expert(x) per route in plan order ([N*k, D]
    bf16, for add_rmsnorm_routed).  path "grouped": tcgen05 GEMMs over the
    plan's tile_m-row tiles; "decode": weight-streaming kernels; "auto": the
    grouped GEMMs when the plan has several rows per expert."""
    n_rows = plan.perm_token.numel()
    e = w13.shape[0]
    if path not in ("auto", "grouped", "decode"):
        raise ValueError(f"unknown expert path {path!r}")
    if path == "decode" or (path == "auto" and not use_grouped_rows(n_rows, e, x.shape[-1],
                                                                    w2.shape[-1])):
        return moe_decode_experts(x, plan, w13, w2, y_rows=y_rows)
    if y_rows is None:
        y_rows = torch.empty(n_rows, x.shape[-1], dtype=torch.bfloat16, device=x.device)
    scratch = torch.empty(grouped_scratch_bytes(n_rows, x.shape[-1], w2.shape[-1]),
                          dtype=torch.uint8, device=x.device)
    moe_grouped_experts_to(x, n_rows, plan.perm_token, plan.perm_prob, plan.offsets,
                           plan.tile_offsets, plan.tile_m, w13, w2, scratch, y_rows)
    return y_rows


def add_rmsnorm_routed(streams: torch.Tensor, y_rows: torch.Tensor, plan: RoutePlan,
                       weight: torch.Tensor | None, eps: float, *,
                       out_bf16: torch.Tensor | None = None, out_f32: torch.Tensor | None = None,
                       normalize: bool = True) -> None:
    """streams += sum_s y_rows[route_pos[t, s]]; then RMSNorm as add_rmsnorm."""
    _require_cuda(streams, y_rows, weight)
    _inplace(streams, "streams")
    d = streams.shape[-1]
    n = streams.numel() // d
    k = plan.topk_idx.shape[1]
    _native.call("llmyb_add_rmsnorm_routed", _ptr(streams), _ptr(y_rows), _ptr(plan.route_pos), k,
                 n, d, _ptr(weight), float(eps), int(normalize), _ptr(out_bf16), _ptr(out_f32),
                 _stream())


def decode_fused_supported(n: int, d: int, e: int, k: int, *k_ins: int) -> bool:
    """Shapes the fused small-batch decode kernels take: up to 8 tokens and 64
    (token, expert) pairs (the last CTA combines N*(2+E) partial sums), D and
    every projection input width a multiple of 8 and at most 2048."""
    return (1 <= n <= 8 and n * e <= 64 and k <= 32 and d % 8 == 0 and d <= 2048
            and all(x % 8 == 0 and 0 < x <= 2048 for x in k_ins))


def decode_norm_gemv(streams_in: torch.Tensor, delta: torch.Tensor | None, plan: RoutePlan | None,
                     norm_w: torch.Tensor, eps: float, w: torch.Tensor, out: torch.Tensor,
                     streams_out: torch.Tensor, normed_out: torch.Tensor | None = None) -> None:
    """[A] streams_out = streams_in + delta (or the routed sum over plan.route_pos);
    out = w . RMSNorm(streams_out) * norm_w (bf16), every CTA normalising for itself."""
    _require_cuda(streams_in, delta, norm_w, w, out, streams_out, normed_out)
    for t_, nm in ((out, "out"), (streams_out, "streams_out")):
        _inplace(t_, nm)
    n, d = streams_in.shape
    route_pos, k = (plan.route_pos, plan.topk_idx.shape[1]) if plan is not None else (None, 0)
    _native.call("llmyb_decode_norm_gemv", _ptr(streams_in), _ptr(delta), _ptr(route_pos), k, n, d,
                 _ptr(norm_w), float(eps), _ptr(w), w.shape[0], _ptr(out), out.stride(0),
                 _ptr(streams_out), _ptr(normed_out), _stream())


def fold_router(w_router: torch.Tensor, ffn_norm: torch.Tensor,
                router_norm: torch.Tensor) -> torch.Tensor:
    """W_r * ffn_norm * router_norm (fp32 [E, D]): the router weights of
    decode_out_router, whose two RMSNorms reduce to per-token scales."""
    return (w_router.float() * ffn_norm.float()[None, :] * router_norm.float()[None, :]).contiguous()


def decode_out_router(inp: torch.Tensor, w: torch.Tensor, streams: torch.Tensor,
                      ffn_norm: torch.Tensor, w_router_folded: torch.Tensor, k: int, eps: float,
                      m_bf: torch.Tensor, counter: torch.Tensor, *,
                      conv_w: torch.Tensor | None = None, normed: torch.Tensor | None = None,
                      history: torch.Tensor | None = None, tile_m: int = TILE_M) -> RoutePlan:
    """[C] mixed = w . inp (+ the GDN conv gate with conv_w / normed / history,
    history rolled); streams += mixed; m_bf = RMSNorm_ffn(streams); routes and
    plan (fold_router weights).  counter: int32 [1] zero word reused across
    calls."""
    _require_cuda(inp, w, streams, ffn_norm, w_router_folded, m_bf, counter, conv_w, normed,
                  history)
    _rows(inp, "inp")
    _inplace(streams, "streams")
    _inplace(m_bf, "m_bf")
    if history is not None:
        _inplace(history, "history")
    n, d = streams.shape
    e = w_router_folded.shape[0]
    dev = streams.device
    idx = torch.empty(n, k, dtype=torch.int64, device=dev)
    prob = torch.empty(n, k, dtype=torch.float32, device=dev)
    b = _plan_buffers(n, e, k, dev, False)
    partials = torch.empty((d + 7) // 8 * n * (2 + e), dtype=torch.float32, device=dev)
    _native.call("llmyb_decode_out_router", _ptr(inp), inp.stride(0), inp.shape[1], _ptr(w), n, d,
                 _ptr(conv_w), _ptr(normed), _ptr(history), _ptr(partials), _ptr(counter),
                 _ptr(streams), _ptr(ffn_norm), _ptr(w_router_folded), float(eps), e, k,
                 int(tile_m), _ptr(m_bf), _ptr(idx), _ptr(prob), _ptr(b["counts"]),
                 _ptr(b["offsets"]), _ptr(b["tile_offsets"]), _ptr(b["perm_token"]),
                 _ptr(b["perm_prob"]), _ptr(b["route_pos"]), _stream())
    return RoutePlan(idx, prob, **b, tile_m=tile_m)


def pack_w13(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """Interleave [E,F,D] gate/up stacks into the [E,2F,D] GEMM1 operand."""
    _require_cuda(w_gate, w_up)
    w_gate = w_gate.to(torch.bfloat16).contiguous()
    w_up = w_up.to(torch.bfloat16).contiguous()
    e, f, d = w_gate.shape
    out = torch.empty(e, 2 * f, d, dtype=torch.bfloat16, device=w_gate.device)
    _native.call("llmyb_moe_pack_w13", _ptr(w_gate), _ptr(w_up), e, f, d, _ptr(out), _stream())
    return out


def moe_grouped(x: torch.Tensor, plan: RoutePlan, w13: torch.Tensor, w2: torch.Tensor,
                out: torch.Tensor | None = None, scratch: torch.Tensor | None = None,
                path: str = "auto") -> torch.Tensor:
    """Routed SwiGLU experts: out[t] = sum_s p_ts * down(silu(gate x_t) * up x_t).

    path "grouped" = tcgen05 grouped GEMM over 128-row expert tiles,
    "decode" = weight-streaming kernels for a few rows per expert, "auto"
    picks "decode" when the average expert sees fewer than 32 rows."""
    _require_cuda(x, w13, w2)
    if x.dtype != torch.bfloat16:
        raise ValueError("moe_grouped computes in bf16")
    x = x.contiguous()
    n, d = x.shape
    k = plan.topk_idx.shape[1]
    e, f2, d2 = w13.shape
    f = f2 // 2
    if d2 != d or tuple(w2.shape) != (e, d, f):
        raise ValueError("expert weight shapes do not match the activations")
    if out is None:
        out = torch.empty(n, d, dtype=torch.bfloat16, device=x.device)
    if path == "auto":
        decode_ok = d <= 2048 and f <= 2048 and d % 128 == 0 and f % 128 == 0
        path = "decode" if decode_ok and (n * k < 32 * e or not grouped_shape_ok(d, f)) \
            else "grouped"
    lib = _native.lib()
    if path == "decode":
        need = int(lib.llmyb_moe_decode_scratch_bytes(n, k, d, f))
    else:
        need = int(lib.llmyb_moe_grouped_scratch_bytes(n, k, d, f))
    if scratch is None or scratch.numel() < need:
        scratch = torch.empty(max(need, 16), dtype=torch.uint8, device=x.device)
    if path == "decode":
        _native.call("llmyb_moe_decode_swiglu", _ptr(x), n, d, k, _ptr(plan.perm_token),
                     _ptr(plan.perm_prob), _ptr(plan.route_pos), _ptr(plan.offsets), e, _ptr(w13),
                     _ptr(w2), f, _ptr(scratch), _ptr(out), _stream())
    else:
        _native.call("llmyb_moe_grouped_swiglu", _ptr(x), n, d, k, _ptr(plan.perm_token),
                     _ptr(plan.perm_prob), _ptr(plan.route_pos), _ptr(plan.offsets),
                     _ptr(plan.tile_offsets), plan.tile_m, e, _ptr(w13), _ptr(w2), f,
                     _ptr(scratch), _ptr(out), _ptr(device_status(x.device)), _stream())
    return out


# ------------------------------------------------------------------- GDN
def _heads_view(t: torch.Tensor, name: str) -> tuple[int, int]:
    """(data pointer, elements between consecutive tokens) of a [..., H, D] view
    whose last two dims are packed and whose tokens are evenly strided."""
    if t.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be bf16")
    if t.stride(-1) != 1 or t.stride(-2) != t.shape[-1]:
        raise ValueError(f"{name}: last two dims must be contiguous")
    tok = t.stride(-3)
    if t.dim() == 4 and t.stride(0) != t.shape[1] * tok:
        raise ValueError(f"{name}: tokens must be evenly strided")
    return t.data_ptr(), tok


def _beta_view(beta: torch.Tensor) -> tuple[int, int]:
    """beta [..., tokens, H] (bf16, heads contiguous) -> (pointer, token stride)."""
    if beta.dtype != torch.bfloat16:
        raise ValueError("beta must be bf16")
    if beta.stride(-1) != 1:
        raise ValueError("beta heads must be contiguous")
    return beta.data_ptr(), beta.stride(-2)


def gdn_activate(proj: torch.Tensor, heads: int, key_dim: int, value_dim: int,
                 beta_bias: torch.Tensor | None) -> None:
    """In place on the fused [N, 2HK+2HV+H] projection: L2-normalise q,k per head,
    sigmoid(gate), sigmoid(beta + bias)  (gated_deltanet.py:128-131)."""
    _require_cuda(proj)
    _inplace(proj, "proj")
    beta_bias = None if beta_bias is None else beta_bias.to(torch.float32).contiguous()
    n = proj.numel() // proj.shape[-1]
    _native.call("llmyb_gdn_activate", _ptr(proj), n, proj.shape[-1], heads, key_dim, value_dim,
                 _ptr(beta_bias), _stream())


def gdn_step(q, k, v, gate, beta, state, *, decay_logit=None, log_alpha=None, reset=None,
             out=None, raw_inputs: bool = False, beta_bias=None):
    """One decode token per row.  q,k [B,H,K]; v,gate [B,H,V]; beta [B,H] (bf16; already
    activated, or raw projections with raw_inputs=True and beta_bias [H]); state
    [B,H,K,V] fp32 updated in place; returns out [B,H,V] bf16."""
    _require_cuda(q, k, v, gate, beta, state)
    bsz, h, kd = q.shape
    vd = v.shape[-1]
    qp, qs = _heads_view(q, "q")
    kp, ks = _heads_view(k, "k")
    vp, vs = _heads_view(v, "v")
    gp, gs = _heads_view(gate, "gate")
    bp, bs = _beta_view(beta)
    if out is None:
        out = torch.empty(bsz, h, vd, dtype=torch.bfloat16, device=q.device)
    if state.dtype != torch.float32 or not state.is_contiguous():
        raise ValueError("state must be contiguous fp32")
    r = None if reset is None else reset.to(torch.uint8).contiguous()
    _inplace(state, "state")
    decay_logit = None if decay_logit is None else decay_logit.to(torch.float32).contiguous()
    log_alpha = None if log_alpha is None else log_alpha.to(torch.float32).contiguous()
    bb = None if beta_bias is None else beta_bias.to(torch.float32).contiguous()
    _native.call("llmyb_gdn_step", qp, qs, kp, ks, vp, vs, gp, gs, bp, bs, _ptr(decay_logit),
                 _ptr(log_alpha), _ptr(r), bsz, h, kd, vd, _ptr(state), _ptr(out),
                 out.stride(-3), int(raw_inputs), _ptr(bb), _stream())
    return out


def gdn_prefill(q, k, v, gate, beta, state, *, decay_logit=None, log_alpha=None, reset=None,
                out=None, scratch=None):
    """Chunked scan over [B,T] tokens.  q,k [B,T,H,K]; v,gate [B,T,H,V]; beta [B,T,H]
    (bf16, activated); state [B,H,K,V] fp32 in/out; returns out [B,T,H,V] bf16."""
    _require_cuda(q, k, v, gate, beta, state)
    bsz, t, h, kd = q.shape
    vd = v.shape[-1]
    qp, qs = _heads_view(q, "q")
    kp, ks = _heads_view(k, "k")
    vp, vs = _heads_view(v, "v")
    gp, gs = _heads_view(gate, "gate")
    bp, bs = _beta_view(beta)
    if out is None:
        out = torch.empty(bsz, t, h, vd, dtype=torch.bfloat16, device=q.device)
    need = int(_native.lib().llmyb_gdn_prefill_scratch_bytes(bsz, t, h, kd, vd))
    if scratch is None or scratch.numel() < need:
        scratch = torch.empty(max(need, 16), dtype=torch.uint8, device=q.device)
    r = None if reset is None else reset.to(torch.uint8).contiguous()
    la = None if log_alpha is None else log_alpha.to(torch.float32).contiguous()
    _inplace(state, "state")
    decay_logit = None if decay_logit is None else decay_logit.to(torch.float32).contiguous()
    _native.call("llmyb_gdn_prefill", qp, qs, kp, ks, vp, vs, gp, gs, bp, bs, _ptr(decay_logit),
                 _ptr(la), _ptr(r), bsz, t, h, kd, vd, _ptr(state), _ptr(out), out.stride(-3),
                 _ptr(scratch), _ptr(device_status(q.device)), _stream())
    return out


def gdn_history_set(x, history) -> None:
    """history [B,3,D] = the last three rows of x [B,T,D] (zero rows when T < 3):
    the decode conv history a prompt leaves (model/model.py:180-182)."""
    _require_cuda(x, history)
    _inplace(history, "history")
    x = x.contiguous()
    bsz, t, d = x.shape
    if tuple(history.shape) != (bsz, 3, d) or history.dtype != torch.bfloat16 or x.dtype != torch.bfloat16:
        raise ValueError("history must be bf16 [B, 3, D] for bf16 x [B, T, D]")
    _native.call("llmyb_gdn_history_set", _ptr(x), _ptr(history), bsz, t, d, _stream())


def zero_regions(regions: torch.Tensor, max_bytes: int) -> None:
    """Zero every (address, bytes) region of the int64 device table regions
    [n, 2] in one launch (see region_table)."""
    _require_cuda(regions)
    if regions.dtype != torch.int64 or regions.dim() != 2 or regions.shape[1] != 2:
        raise ValueError("regions must be an int64 [n, 2] table of (address, bytes)")
    _native.call("llmyb_zero_regions", _ptr(regions.contiguous()), regions.shape[0],
                 int(max_bytes), _stream())


def region_table(tensors, device) -> tuple[torch.Tensor, int]:
    """(int64 device table [n, 2] of (address, bytes), largest size) for the
    contiguous tensors, to zero them all with zero_regions."""
    rows = []
    for t in tensors:
        if not t.is_contiguous():
            raise ValueError("region_table takes contiguous tensors")
        if t.numel():
            rows.append((t.data_ptr(), t.numel() * t.element_size()))
    table = torch.tensor(rows if rows else [(0, 0)], dtype=torch.int64).to(device)
    return table[: len(rows)], max((r[1] for r in rows), default=0)


def gdn_conv_gate(x, y_proj, conv_w, *, history=None, reset=None, out=None, residual=None,
                  roll_history=False):
    """y = y_proj * sigmoid(causal_conv4(x)); into `out` or added into `residual`."""
    _require_cuda(x, y_proj, conv_w)
    x, y_proj = x.contiguous(), y_proj.contiguous()
    if history is not None:
        _inplace(history, "history")
    if residual is not None:
        _inplace(residual, "residual")
    bsz, t, d = x.shape
    w = conv_w.reshape(d, -1).to(torch.float32).contiguous()
    if out is None and residual is None:
        out = torch.empty_like(y_proj)
    r = None if reset is None else reset.to(torch.uint8).contiguous()
    _native.call("llmyb_gdn_conv_gate", _ptr(x), _ptr(y_proj), _ptr(w), _ptr(history), _ptr(r),
                 bsz, t, d, _ptr(out), _ptr(residual), int(roll_history), _stream())
    return residual if residual is not None else out


# ------------------------------------------------------ banded attention
def _tokens(t: torch.Tensor, name: str) -> tuple[int, int]:
    """(pointer, token stride) of a bf16 [B, T, ...] tensor whose per-token
    block is packed and whose tokens are evenly strided."""
    if t.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be bf16")
    inner = 1
    for dim in range(t.dim() - 1, 1, -1):
        if t.stride(dim) != inner:
            raise ValueError(f"{name}: per-token block must be contiguous")
        inner *= t.shape[dim]
    if t.stride(0) != t.shape[1] * t.stride(1):
        raise ValueError(f"{name}: tokens must be evenly strided")
    return t.data_ptr(), t.stride(1)


def banded_attention(q, k, v, window: int, scale: float | None = None, out=None):
    """Per-head causal sliding-window attention (sample_standalone.py:70-85):
    q,k [B,T,H,D]; v [B,T,H or 1,D] -> [B,T,H,D] bf16."""
    _require_cuda(q, k, v)
    bsz, t, h, d = q.shape
    qp, qs = _tokens(q, "q")
    kp, ks = _tokens(k, "k")
    vp, vs = _tokens(v, "v")
    if out is None:
        out = torch.empty(bsz, t, h, d, dtype=torch.bfloat16, device=q.device)
    scale = d ** -0.5 if scale is None else float(scale)
    _native.call("llmyb_banded_attention", qp, qs, kp, ks, vp, vs, v.shape[2], bsz, t, h, d,
                 int(window), scale, _ptr(out), out.stride(1), _ptr(device_status(q.device)),
                 _stream())
    return out


def csa_local_prefill(q, k, v, window: int, out=None):
    """CSA local branch (csa.py:42-75): q,k [B,T,H,Dh]; v [B,T,D] -> [B,T,D]."""
    _require_cuda(q, k, v)
    bsz, t, h, dh = q.shape
    dm = v.shape[-1]
    qp, qs = _tokens(q, "q")
    kp, ks = _tokens(k, "k")
    vp, vs = _tokens(v, "v")
    if out is None:
        out = torch.empty(bsz, t, dm, dtype=torch.bfloat16, device=q.device)
    need = int(_native.lib().llmyb_csa_prefill_scratch_bytes(bsz, t, h, int(window)))
    scratch = torch.empty(max(need, 16), dtype=torch.uint8, device=q.device)
    _native.call("llmyb_csa_local_prefill", qp, qs, kp, ks, vp, vs, bsz, t, h, dh, dm, int(window),
                 _ptr(out), out.stride(1), _ptr(scratch), _ptr(device_status(q.device)), _stream())
    return out


def csa_ring_write(k, v, kcache, vcache) -> None:
    """Decode ring caches after a prompt (csa.py:208-258 layout): token p of the
    last min(T, W) tokens of k [B,T,kw] and v [B,T,vw] (evenly strided token
    rows, e.g. column slices of the fused projection) into slot p % W of
    kcache [B,W,kw] and vcache [B,W,vw]; the other slots keep their rows."""
    _require_cuda(k, v, kcache, vcache)
    _inplace(kcache, "kcache")
    _inplace(vcache, "vcache")
    bsz, t, kw = k.shape
    vw = v.shape[-1]
    w = kcache.shape[1]
    if tuple(kcache.shape) != (bsz, w, kw) or tuple(vcache.shape) != (bsz, w, vw):
        raise ValueError("kcache / vcache must be [B, W, width] for the k / v widths")
    if kcache.dtype != torch.bfloat16 or vcache.dtype != torch.bfloat16:
        raise ValueError("ring caches must be bf16")
    kp, ks = _tokens(k, "k")
    vp, vs = _tokens(v, "v")
    _native.call("llmyb_csa_ring_write", kp, ks, vp, vs, bsz, t, kw, vw, _ptr(kcache),
                 _ptr(vcache), w, _stream())


def csa_local_decode(q, knew, vnew, kcache, vcache, positions, heads: int, out=None):
    """CSA decode (csa.py:172-206) over a ring K/V cache: q,knew [B,H*Dh]; vnew [B,D];
    kcache [B,W,H*Dh]; vcache [B,W,D]; positions [B] int32 = position of the new
    token, whose K/V are written to slot position % W.  Returns [B,D] bf16."""
    _require_cuda(q, knew, vnew, kcache, vcache, positions)
    for t_, nm in ((q, "q"), (knew, "knew"), (vnew, "vnew")):
        _rows(t_, nm)
    _inplace(kcache, "kcache")
    _inplace(vcache, "vcache")
    positions = positions.contiguous()
    bsz, hd = q.shape
    dm = vnew.shape[-1]
    w = kcache.shape[1]
    if positions.dtype != torch.int32:
        raise ValueError("positions must be int32")
    if out is None:
        out = torch.empty(bsz, dm, dtype=torch.bfloat16, device=q.device)
    _native.call("llmyb_csa_local_decode", _ptr(q), q.stride(0), _ptr(knew), knew.stride(0),
                 _ptr(vnew), vnew.stride(0), _ptr(kcache), _ptr(vcache), _ptr(positions), bsz,
                 heads, hd // heads, dm, w, _ptr(out), out.stride(0),
                 _ptr(device_status(q.device)), _stream())
    return out


# ------------------------------------------------------------- sampling
def seen_bitmask(generated: list[list[int]], vocab: int, device) -> torch.Tensor:
    """[B, ceil(V/32)] int32 bitmask of the ids in each row's generated list."""
    words = (vocab + 31) // 32
    mask = torch.zeros(len(generated), words * 32, dtype=torch.bool)
    for r, ids in enumerate(generated):
        if ids:
            mask[r, torch.tensor(sorted(set(int(i) for i in ids)), dtype=torch.long)] = True
    bits = (mask.view(len(generated), words, 32).to(torch.int64)
            << torch.arange(32, dtype=torch.int64)).sum(-1)
    return bits.to(torch.uint32).view(torch.int32).to(device)


def sample(logits: torch.Tensor, *, temperature: float, top_k: int, top_p: float,
           repetition_penalty: float = 1.0, seen: torch.Tensor | None = None,
           blocked: torch.Tensor | None = None, uniforms: torch.Tensor | None = None,
           update_seen: bool = False, out: torch.Tensor | None = None,
           logprob: torch.Tensor | None = None):
    """Device sampler (sample_standalone.py:5383-5423 semantics, inverse-CDF draw at
    `uniforms`).  Returns (tokens [B] int64, raw log-prob of each token [B] fp32)."""
    _require_cuda(logits, seen, blocked, uniforms)
    if logits.dtype != torch.float32 or logits.stride(-1) != 1:
        raise ValueError("logits must be fp32 with a contiguous vocabulary dim")
    if seen is not None:
        _inplace(seen, "seen")
    if blocked is not None:
        blocked = blocked.to(torch.int32).contiguous()
    if uniforms is not None:
        uniforms = uniforms.to(torch.float32).contiguous()
    bsz, vocab = logits.shape
    if uniforms is None and temperature > 1e-4:
        uniforms = torch.rand(bsz, device=logits.device)
    if out is None:
        out = torch.empty(bsz, dtype=torch.int64, device=logits.device)
    if logprob is None:
        logprob = torch.empty(bsz, dtype=torch.float32, device=logits.device)
    nb = 0 if blocked is None else blocked.numel()
    _native.call("llmyb_sample", _ptr(logits), logits.stride(0), bsz, vocab, _ptr(seen),
                 0 if seen is None else seen.stride(0), float(repetition_penalty), _ptr(blocked),
                 nb, float(temperature), int(top_k), float(top_p), _ptr(uniforms), _ptr(out),
                 _ptr(logprob), int(update_seen), _ptr(device_status(logits.device)), _stream())
    return out, logprob


# ------------------------------------------------------- residual stream
def embed(ids: torch.Tensor, table: torch.Tensor, stream_seed: torch.Tensor | None,
          out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 residual stream = table[ids] + stream_seed (model/model.py:442-444)."""
    _require_cuda(ids, table, stream_seed)
    ids = ids.to(torch.int64).contiguous()
    table = table.contiguous()
    n = ids.numel()
    d = table.shape[1]
    if out is None:
        out = torch.empty(*ids.shape, d, dtype=torch.float32, device=ids.device)
    _native.call("llmyb_embed", _ptr(ids), n, _ptr(table), table.shape[0], d, _ptr(stream_seed),
                 _ptr(out), _ptr(device_status(ids.device)), _stream())
    return out


def add_rmsnorm(streams: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor | None,
                eps: float, *, out_bf16: torch.Tensor | None = None,
                out_f32: torch.Tensor | None = None, normalize: bool = True) -> None:
    """streams (fp32) += delta (bf16, optional); write RMSNorm(streams) * weight
    (norms.py:13-16) as bf16 and/or fp32."""
    _require_cuda(streams, delta, weight)
    _inplace(streams, "streams")
    delta = None if delta is None else delta.contiguous()
    for o, nm in ((out_bf16, "out_bf16"), (out_f32, "out_f32")):
        if o is not None:
            _inplace(o, nm)
    d = streams.shape[-1]
    n = streams.numel() // d
    _native.call("llmyb_add_rmsnorm", _ptr(streams), _ptr(delta), n, d, _ptr(weight), float(eps),
                 int(normalize), _ptr(out_bf16), _ptr(out_f32), _stream())


def add_rmsnorm_router(streams: torch.Tensor, delta: torch.Tensor | None,
                       ffn_weight: torch.Tensor, router_weight: torch.Tensor, eps: float, *,
                       out_bf16: torch.Tensor | None, router_in: torch.Tensor) -> None:
    """streams += delta; m = RMSNorm(streams) * ffn_weight (bf16 into out_bf16);
    router_in = RMSNorm(m) * router_weight (fp32), in one pass: the same bits as
    add_rmsnorm(..., out_f32=m) followed by add_rmsnorm(m, None, router_weight)."""
    _require_cuda(streams, delta, ffn_weight, router_weight)
    _inplace(streams, "streams")
    _inplace(router_in, "router_in")
    if out_bf16 is not None:
        _inplace(out_bf16, "out_bf16")
    delta = None if delta is None else delta.contiguous()
    d = streams.shape[-1]
    n = streams.numel() // d
    _native.call("llmyb_add_rmsnorm_router", _ptr(streams), _ptr(delta), n, d, _ptr(ffn_weight),
                 _ptr(router_weight), float(eps), _ptr(out_bf16), _ptr(router_in), _stream())


def add_rmsnorm_router_supported(d_model: int) -> bool:
    return d_model % 8 == 0 and d_model <= 8192


def rmsnorm_bf16(x: torch.Tensor, weight: torch.Tensor | None, eps: float,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    _require_cuda(x, weight)
    x = x.contiguous()
    d = x.shape[-1]
    if out is None:
        out = torch.empty_like(x)
    _inplace(out, "out")
    _native.call("llmyb_rmsnorm_bf16", _ptr(x), x.numel() // d, d, _ptr(weight), float(eps),
                 _ptr(out), _stream())
    return out


# ------------------------------------------------------------ engine device ops
def mhc_sinkhorn4(logits: torch.Tensor, iterations: int = 20,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Sinkhorn-normalised exp of fp32 [..., 4, 4] matrices (mhc.py:12-17):
    `iterations` rounds of row then column log-normalisation."""
    _require_cuda(logits, out)
    if logits.dtype != torch.float32 or tuple(logits.shape[-2:]) != (4, 4):
        raise ValueError("mhc_sinkhorn4 takes fp32 [..., 4, 4] matrices")
    x = logits.contiguous()
    if out is None:
        out = torch.empty_like(x)
    elif not out.is_contiguous() or out.shape != x.shape or out.dtype != torch.float32:
        raise ValueError("out must be a contiguous fp32 tensor of the input's shape")
    n = x.numel() // 16
    if n == 0:
        return out
    _native.call("llmyb_mhc_sinkhorn4", _ptr(x), _ptr(out), n, int(iterations), _stream())
    return out


def moe_selected_fp32(x: torch.Tensor, idx: torch.Tensor, prob: torch.Tensor,
                      gate_up: torch.Tensor, down: torch.Tensor) -> torch.Tensor:
    """One token through its k routed experts, fp32 (llmy_moe_selected_fp32):
    x [D], idx [k] int64, prob [k], gate_up [E, 2H, D] (gate rows then up rows),
    down [E, D, H].  Returns out [D]."""
    _require_cuda(x, idx, prob, gate_up, down)
    e, h2, d = gate_up.shape
    h = h2 // 2
    k = idx.numel()
    if (x.numel() != d or tuple(down.shape) != (e, d, h) or prob.numel() != k
            or idx.dtype != torch.int64 or x.dtype != torch.float32
            or gate_up.dtype != torch.float32 or down.dtype != torch.float32
            or prob.dtype != torch.float32):
        raise ValueError("moe_selected_fp32: shapes or dtypes do not match")
    x, idx, prob = x.contiguous(), idx.contiguous(), prob.contiguous()
    gate_up, down = gate_up.contiguous(), down.contiguous()
    act = torch.empty(k, h, dtype=torch.float32, device=x.device)
    route = torch.empty(k, d, dtype=torch.float32, device=x.device)
    out = torch.empty(d, dtype=torch.float32, device=x.device)
    _native.call("llmyb_moe_selected_fp32", _ptr(x), _ptr(idx), _ptr(prob), _ptr(gate_up),
                 _ptr(down), _ptr(act), _ptr(route), _ptr(out), d, h, e, k, _stream())
    return out


# --------------------------------------------------------- hyper-connections
_ZEROS: dict = {}


def _zero_scalar(device: torch.device) -> torch.Tensor:
    z = _ZEROS.get(device)
    if z is None:
        z = _ZEROS[device] = torch.zeros(4, dtype=torch.float32, device=device)
    return z


def mhc_read(streams: torch.Tensor, n_streams: int, mhc, norm_w: torch.Tensor | None, eps: float,
             iterations: int, maps: torch.Tensor, *, out_bf16: torch.Tensor | None = None,
             out_f32: torch.Tensor | None = None) -> None:
    """Sub-layer input from the S residual streams (mhc.py:135-156, :193-206):
    streams [N, S*D] fp32; mhc a weights.MhcBlock; writes the maps [N, 2S+S*S]
    and RMSNorm(LayerNorm(sum_s pre_s stream_s)) * norm_w into out_bf16 / out_f32."""
    _require_cuda(streams, maps, out_bf16, out_f32)
    n = streams.shape[0]
    d = streams.shape[1] // n_streams
    if getattr(mhc, "static", False):
        # an all-zero theta gives zero logits: one zero read for every map
        raw, ld_tok, ld_map = _zero_scalar(streams.device), 0, 0
    else:
        raw = torch.mm(streams, mhc.theta.t())  # theta with the mapping-norm weight folded in
        ld_tok, ld_map = raw.stride(0), raw.stride(1)
    _native.call("llmyb_mhc_read", _ptr(streams), n, n_streams, d, _ptr(raw), ld_tok, ld_map,
                 _ptr(mhc.bias),
                 _ptr(mhc.scalars), _ptr(mhc.ln_w), _ptr(mhc.ln_b), _ptr(norm_w), float(eps),
                 int(iterations), _ptr(maps), _ptr(out_bf16), _ptr(out_f32), _stream())


def mhc_write(streams: torch.Tensor, n_streams: int, mhc, maps: torch.Tensor,
              delta: torch.Tensor | None, plan: RoutePlan | None = None) -> None:
    """streams [N, S*D] += g * scale * (res @ streams + post * update) in place
    (mhc.py:208-229); update = delta [N, D] bf16, or with `plan` the sum of
    each token's routed expert rows delta[plan.route_pos[t*k + s]]."""
    _require_cuda(streams, maps, delta)
    _inplace(streams, "streams")
    n = streams.shape[0]
    d = streams.shape[1] // n_streams
    route_pos, k = (None, 0)
    if plan is not None:
        route_pos, k = plan.route_pos, plan.topk_idx.shape[1]
    if delta is not None:
        delta = delta.contiguous()
    _native.call("llmyb_mhc_write", _ptr(streams), n, n_streams, d, _ptr(delta), _ptr(route_pos),
                 int(k), _ptr(maps), _ptr(mhc.stream_scale), _ptr(mhc.scalars), _stream())


# ----------------------------------------------------- router local context
def router_context_logits(r_in: torch.Tensor, moe, window: int, *, batch: int, seq: int,
                          ring: torch.Tensor | None = None,
                          positions: torch.Tensor | None = None) -> torch.Tensor:
    """Router logits with the ContextAwareRouter's local context
    (context_router.py:59-74 / :89-133): router (local + g ctx(box)) with box
    the causal window mean of LayerNorm(down(local)).  r_in [batch*seq, D]
    fp32 is the router-normed input; moe a weights.MoeBlock with the ctx_*
    fields.  Prefill (positions None): the window runs over each row's `seq`
    tokens and the last `window` latents go to `ring` [batch, window, L]; decode
    (seq 1, positions [batch]): the new latent enters the ring first."""
    _require_cuda(r_in, ring, positions)
    lat = torch.mm(r_in, moe.ctx_down.t())
    box = torch.empty_like(lat)
    latent = lat.shape[1]
    if positions is None:
        _native.call("llmyb_router_ctx_prefill", _ptr(lat), int(batch), int(seq), latent,
                     int(window), _ptr(moe.ctx_ln_w), _ptr(moe.ctx_ln_b), _ptr(box), _ptr(ring),
                     _stream())
    else:
        _native.call("llmyb_router_ctx_step", _ptr(lat), int(batch), latent, int(window),
                     _ptr(moe.ctx_ln_w), _ptr(moe.ctx_ln_b), _ptr(ring), _ptr(positions),
                     _ptr(box), _stream())
    logits = torch.mm(r_in, moe.router.t())
    return logits.addmm_(box, moe.ctx_logits.t(), alpha=moe.ctx_gate)


# ------------------------------------------------------------- shared experts
def plan_append_shared(plan: RoutePlan, n_shared: int) -> RoutePlan:
    """The plan extended by n_shared shared experts (moe.py:185-198, :221-234)
    as plan experts E..E+n-1 that every token is routed to with probability
    1/sqrt(n), their rows after the routed ones (expert E+s holds tokens
    0..N-1 at rows N*k + s*N + t): the expert kernels scale each row by that
    probability and the combine over a token's k + n rows gives routed +
    sum_s SwiGLU_s(x) / sqrt(n).  Expert weights must be stacked routed first,
    then shared.  One kernel launch, no synchronisation."""
    n = int(n_shared)
    if n <= 0:
        return plan
    _require_cuda(plan.offsets)
    tokens, k = plan.topk_idx.shape
    e = plan.n_experts
    out = _plan_buffers(tokens, e + n, 1, plan.offsets.device, False)
    rows = tokens * (k + n)
    dev = plan.offsets.device
    i32 = dict(dtype=torch.int32, device=dev)
    out.update(perm_token=torch.empty(rows, **i32), route_pos=torch.empty(rows, **i32),
               perm_prob=torch.empty(rows, dtype=torch.float32, device=dev))
    idx = torch.empty(tokens, k + n, dtype=torch.int64, device=dev)
    prob = torch.empty(tokens, k + n, dtype=torch.float32, device=dev)
    _native.call("llmyb_plan_append_shared", tokens, e, k, n, plan.tile_m, _ptr(plan.topk_idx),
                 _ptr(plan.topk_prob), _ptr(plan.counts), _ptr(plan.offsets),
                 _ptr(plan.tile_offsets), _ptr(plan.perm_token), _ptr(plan.perm_prob),
                 _ptr(plan.route_pos), _ptr(idx), _ptr(prob), _ptr(out["counts"]),
                 _ptr(out["offsets"]), _ptr(out["tile_offsets"]), _ptr(out["perm_token"]),
                 _ptr(out["perm_prob"]), _ptr(out["route_pos"]), _stream())
    return RoutePlan(topk_idx=idx, topk_prob=prob, counts=out["counts"], offsets=out["offsets"],
                     tile_offsets=out["tile_offsets"], perm_token=out["perm_token"],
                     perm_prob=out["perm_prob"], route_pos=out["route_pos"], sort_order=None,
                     tile_m=plan.tile_m)


# ------------------------------------------------------------- loop memory
def loop_mem_norm(x: torch.Tensor, n_streams: int, width: int, ln_w: torch.Tensor | None = None,
                  ln_b: torch.Tensor | None = None, eps: float = 1e-5,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Per token: the mean of the n_streams width-wide fp32 streams of x
    [N, n_streams*width], then LayerNorm(ln_w, ln_b, eps) if ln_w is given."""
    _require_cuda(x, ln_w, ln_b, out)
    if x.dtype != torch.float32 or x.dim() != 2 or x.shape[1] < n_streams * width:
        raise ValueError("loop_mem_norm expects fp32 rows of n_streams * width values")
    _rows(x, "x")
    n = x.shape[0]
    if out is None:
        out = torch.empty(n, width, dtype=torch.float32, device=x.device)
    _rows(out, "out")
    _native.call("llmyb_loop_mem_norm", _ptr(x), x.stride(0), n, int(n_streams), int(width),
                 _ptr(ln_w), _ptr(ln_b), float(eps), _ptr(out), out.stride(0), _stream())
    return out


def loop_mem_attend(q: torch.Tensor, kv: torch.Tensor, n_mem: int, heads: int, head_dim: int,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """Per (token, head) softmax over the n_mem endpoints of q.k/sqrt(hd), times
    v: q [N, H*hd], kv [>= n_mem, N, 2*H*hd] fp32 -> [N, H*hd] fp32."""
    _require_cuda(q, kv, out)
    q, kv = q.contiguous(), kv.contiguous()
    n = q.shape[0]
    if out is None:
        out = torch.empty(n, heads * head_dim, dtype=torch.float32, device=q.device)
    _native.call("llmyb_loop_mem_attend", _ptr(q), _ptr(kv), n, int(n_mem), int(heads),
                 int(head_dim), _ptr(_inplace(out, "out")), _stream())
    return out


def loop_mem_add(streams: torch.Tensor, n_streams: int, delta: torch.Tensor, gate: float) -> None:
    """streams [N, S*D] += gate * delta [N, D] on every stream (fp32, in place)."""
    _require_cuda(streams, delta)
    _inplace(streams, "streams")
    delta = delta.contiguous()
    n, d = delta.shape
    _native.call("llmyb_loop_mem_add", _ptr(streams), n, int(n_streams), d, _ptr(delta),
                 float(gate), _stream())


# ------------------------------------------------------------- CSA remote branch
def csa_remote_prefill(x: torch.Tensor, q: torch.Tensor, w_comp: torch.Tensor, ratio: int,
                       top_k: int, heads: int, pend_sum: torch.Tensor, pend_cnt: torch.Tensor):
    """CSA remote branch over a prompt (csa.py:77-131, compressed_attention.py:85-149).

    x [B, T, D] bf16 (the CSA input), q [B, T, H*Dh] bf16 (a view is fine),
    w_comp [H*Dh + D, D] bf16 = [compressor.key; compressor.value].  Returns
    (remote [B, T, D] bf16, summaries [B, n, H*Dh + D] bf16 = key | value of
    every complete block); pend_sum [B, D] fp32 / pend_cnt [B] int32 receive
    the pending partial block."""
    _require_cuda(x, q, w_comp, pend_sum, pend_cnt)
    bsz, t, d = x.shape
    hd = q.shape[-1]
    n = t // ratio
    _rows(x, "x")
    _rows(q, "q")
    dev = x.device
    means = torch.empty(bsz, max(n, 1), d, dtype=torch.bfloat16, device=dev)
    _native.call("llmyb_csa_block_means", _ptr(x), x.stride(1), bsz, t, d, int(ratio),
                 _ptr(means), _ptr(_inplace(pend_sum, "pend_sum")),
                 _ptr(_inplace(pend_cnt, "pend_cnt")), _stream())
    remote = torch.zeros(bsz, t, d, dtype=torch.bfloat16, device=dev)
    if n == 0:
        return remote, torch.empty(bsz, 0, hd + d, dtype=torch.bfloat16, device=dev)
    summ = torch.mm(means.view(bsz * n, d), w_comp.t()).view(bsz, n, hd + d)
    ldp = (n + 7) // 8 * 8
    p = torch.empty(bsz, t, ldp, dtype=torch.bfloat16, device=dev)
    _native.call("llmyb_csa_remote_rows", _ptr(q), q.stride(1), _ptr(summ), hd + d, bsz, t,
                 int(heads), hd // heads, n, int(ratio), int(top_k), _ptr(p), ldp, _stream())
    torch.bmm(p[..., :n], summ[..., hd:], out=remote)
    return remote, summ


def csa_remote_step(x: torch.Tensor, q: torch.Tensor, w_comp: torch.Tensor, ratio: int,
                    top_k: int, heads: int, mem_k: torch.Tensor, mem_v: torch.Tensor,
                    mem_count: torch.Tensor, pend_sum: torch.Tensor, pend_cnt: torch.Tensor,
                    out: torch.Tensor, scratch: tuple[torch.Tensor, torch.Tensor] | None = None):
    """One decode token of the CSA remote branch (csa.py:208-256,
    compressed_attention.py:151-206): x [B, D] bf16 joins the pending block
    (a completed block's summary is stored at slot mem_count); out [B, D]
    (a row view is fine) receives the remote attention of q [B, H*Dh] over
    the row's summaries.  mem_k [B, cap, H*Dh], mem_v [B, cap, D] bf16."""
    _require_cuda(x, q, w_comp, mem_k, mem_v, mem_count, pend_sum, pend_cnt, out)
    for t_, nm in ((x, "x"), (q, "q"), (out, "out")):
        _rows(t_, nm)
    bsz, d = x.shape
    hd = q.shape[-1]
    cap = mem_k.shape[1]
    if scratch is None:
        scratch = (torch.empty(bsz * heads * top_k, dtype=torch.int32, device=x.device),
                   torch.empty(bsz * heads * top_k, dtype=torch.float32, device=x.device))
    _native.call("llmyb_csa_remote_step", _ptr(x), x.stride(0), _ptr(q), q.stride(0), bsz,
                 int(heads), hd // heads, d, int(ratio), int(top_k), cap, _ptr(w_comp),
                 _ptr(_inplace(mem_k, "mem_k")), _ptr(_inplace(mem_v, "mem_v")),
                 _ptr(_inplace(mem_count, "mem_count")), _ptr(_inplace(pend_sum, "pend_sum")),
                 _ptr(_inplace(pend_cnt, "pend_cnt")), _ptr(scratch[0]), _ptr(scratch[1]),
                 _ptr(out), out.stride(0), _ptr(device_status(x.device)), _stream())
    return out
