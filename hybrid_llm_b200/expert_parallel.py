"""Expert parallelism: the routed experts sharded over the ranks of a process group.

The reference runs every expert on one device (model/layers/moe.py:29-82).
Here rank q of W holds experts [q*El, (q+1)*El) (El = E / W), token rows stay
on the rank that owns their sequence (the attention / GDN mixers run data
parallel), and each MoE call moves the routed rows to the experts and the
expert outputs back:

    plan  = kernels.route(...)                       local routing, all E experts
    y, rp = ep.run(x, plan, w13_local, w2_local)     dispatch, experts, return
    kernels.add_rmsnorm_routed(streams, y, replace(plan, route_pos=rp), ...)

``run`` packs W fixed-size dispatch segments (capacity C = max_tokens * k
rows each, so no sizes travel to the host and the step can be replayed as a
CUDA graph), exchanges them, builds the expert-ordered plan of the received
rows, runs the local experts with their outputs written straight into the
return segments, and exchanges those back.  Two exchanges:

* ``"nccl"``: ``all_to_all_single`` of the segments (the baseline);
* ``"p2p"``: every rank maps the others' receive / return buffers (CUDA IPC,
  one process per GPU on one node); the pack kernel stores each segment
  straight into its destination over NVLink and the return kernel stores the
  expert outputs back, each send published by a per-round flag that the
  receiving kernel waits on (bounded).  No collective call is left in the
  step, so it can be captured in a CUDA graph.  The combine is the routed residual add of the next block.  For a
route the expert math, its rounding and the order of the k-term sum are those
of the single-device path, so results are identical for any W.

``ops`` supplies the four device steps; the default runs the llmyb CUDA
kernels and raises for CPU tensors (there is no CPU fallback).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace

import torch
import torch.distributed as dist

from . import _native, kernels


class _CudaMemory:
    """Device memory seen through __cuda_array_interface__ (bytes), so that a
    buffer allocated by the library can be viewed as a torch tensor."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 2, "strides": None}


class PeerBuffers:
    """One CUDA-IPC buffer per rank, mapped by every other rank of the group.

    Layout: receive segments [W, H+C, D] bf16 | return segments [W, C, D] bf16
    | dispatch flags [W] int32 | return flags [W] int32.  Collective: every
    rank constructs it together (handles travel through the process group)."""

    def __init__(self, world: int, rank: int, seg_rows: int, capacity: int, d_model: int,
                 device: torch.device, group=None):
        self.world, self.rank = world, rank
        al = lambda b: (b + 255) // 256 * 256
        self.recv_bytes = world * seg_rows * d_model * 2
        self.ret_off = al(self.recv_bytes)
        self.flags_off = self.ret_off + al(world * capacity * d_model * 2)
        self.nbytes = self.flags_off + al(2 * world * 4)
        lib = _native.lib()
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        _native.check(lib.llmyb_ep_shared_alloc(self.nbytes, ctypes.addressof(ptr),
                                                ctypes.addressof(handle)), "llmyb_ep_shared_alloc")
        self.base = ptr.value
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.peer_base = []
        self._opened = []
        for q in range(world):
            if q == rank:
                self.peer_base.append(self.base)
                continue
            h = (ctypes.c_char * 64).from_buffer_copy(handles[q])
            pp = ctypes.c_void_p()
            _native.check(lib.llmyb_ep_shared_open(ctypes.addressof(h), ctypes.addressof(pp)),
                          "llmyb_ep_shared_open")
            self.peer_base.append(pp.value)
            self._opened.append(pp.value)
        mem = torch.as_tensor(_CudaMemory(self.base, self.nbytes), device=device)
        self.local = mem  # keeps the view object alive
        self.recv = mem[:self.recv_bytes].view(torch.bfloat16).view(world * seg_rows, d_model)
        self.ret_recv = mem[self.ret_off:self.ret_off + world * capacity * d_model * 2].view(
            torch.bfloat16).view(world * capacity, d_model)
        flags = mem[self.flags_off:self.flags_off + 2 * world * 4].view(torch.int32)
        self.dispatch_flags, self.return_flags = flags[:world], flags[world:]
        # host tables of peer addresses (this rank's slots in every peer's buffer)
        vp = ctypes.c_void_p * world
        self.dispatch_segs = vp(*[b + rank * seg_rows * d_model * 2 for b in self.peer_base])
        self.dispatch_flag_ptrs = vp(*[b + self.flags_off + rank * 4 for b in self.peer_base])
        self.return_segs = vp(*[b + self.ret_off + rank * capacity * d_model * 2
                                for b in self.peer_base])
        self.return_flag_ptrs = vp(*[b + self.flags_off + (world + rank) * 4
                                     for b in self.peer_base])

    def close(self) -> None:
        lib = _native.lib()
        for p in self._opened:
            lib.llmyb_ep_shared_close(p)
        self._opened = []
        if self.base:
            torch.cuda.synchronize()
            self.recv = self.ret_recv = self.local = None
            lib.llmyb_ep_shared_free(self.base)
            self.base = 0


class CudaEpOps:
    """The device steps of an expert-parallel MoE call (csrc/ep.cu, moe_gemm.cu,
    moe_decode.cu); each takes the ExpertParallel whose buffers it fills."""

    header_rows = staticmethod(kernels.ep_header_rows)

    @staticmethod
    def scratch_bytes(ep: "ExpertParallel") -> int:
        # the grouped path's scratch also covers the decode kernels' [rows, F]
        return kernels.grouped_scratch_bytes(ep.world * ep.capacity, ep.d_model, ep.ffn)

    @staticmethod
    def dispatch_pack(ep: "ExpertParallel", x, plan, ret_route_pos) -> None:
        if ep.peers is not None:
            pb = ep.peers
            kernels.ep_dispatch_p2p(x, plan, ep.n_experts, ep.world, ep.capacity,
                                    ctypes.addressof(pb.dispatch_segs),
                                    ctypes.addressof(pb.dispatch_flag_ptrs), ep.sync,
                                    ret_route_pos)
        else:
            kernels.ep_dispatch_pack(x, plan, ep.n_experts, ep.world, ep.capacity, ep.send,
                                     ret_route_pos)

    @staticmethod
    def recv_plan(ep: "ExpertParallel") -> None:
        wait = ep.peers.dispatch_flags if ep.peers is not None else None
        kernels.ep_recv_plan(ep.recv, ep.world, ep.capacity, ep.experts_per_rank, ep.offsets_l,
                             ep.perm_token_l, ep.perm_prob_l, ep.out_row,
                             tile_offsets_l=ep.tile_offsets_l, tile_m=ep.tile_m,
                             wait_flags=wait, sync=ep.sync if wait is not None else None)

    @staticmethod
    def return_push(ep: "ExpertParallel") -> None:
        pb = ep.peers
        kernels.ep_return_p2p(ep.ret_send, ep.recv, ep.world, ep.capacity, ep.experts_per_rank,
                              ctypes.addressof(pb.return_segs),
                              ctypes.addressof(pb.return_flag_ptrs), ep.sync)
        kernels.ep_wait(pb.return_flags, ep.world, ep.sync)

    @staticmethod
    def experts_to(ep: "ExpertParallel", w13, w2, grouped: bool) -> None:
        rows = ep.world * ep.capacity
        if grouped:
            kernels.moe_grouped_experts_to(ep.recv, rows, ep.perm_token_l, ep.perm_prob_l,
                                           ep.offsets_l, ep.tile_offsets_l, ep.tile_m, w13, w2,
                                           ep.scratch, ep.ret_send, ep.out_row)
        else:
            kernels.moe_decode_experts_to(ep.recv, rows, ep.perm_token_l, ep.perm_prob_l,
                                          ep.offsets_l, w13, w2, ep.scratch.view(torch.bfloat16),
                                          ep.ret_send, ep.out_row)


@dataclass
class EpResult:
    y_rows: torch.Tensor      # [W*C, D] bf16: expert outputs of this rank's routes
    route_pos: torch.Tensor   # [n_routes] int32: row of y_rows for route t*k+s

    def plan_for_combine(self, plan: kernels.RoutePlan) -> kernels.RoutePlan:
        return replace(plan, route_pos=self.route_pos)


class ExpertParallel:
    """Buffers and call sequence of expert-parallel MoE calls on one rank.

    n_experts: E (divisible by the world size); top_k: k; max_tokens: the most
    tokens this rank routes in one call (sets the capacity C = max_tokens * k).
    """

    def __init__(self, n_experts: int, top_k: int, d_model: int, ffn: int, max_tokens: int, *,
                 group: dist.ProcessGroup | None = None, device: torch.device | str | None = None,
                 ops=None, exchange: str = "nccl"):
        if not dist.is_initialized():
            raise RuntimeError("ExpertParallel needs an initialised torch.distributed group")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_experts % self.world != 0:
            raise ValueError(f"{n_experts} experts do not split over {self.world} ranks")
        self.n_experts, self.top_k, self.d_model, self.ffn = n_experts, top_k, d_model, ffn
        self.experts_per_rank = n_experts // self.world
        self.capacity = int(max_tokens) * int(top_k)
        self.ops = CudaEpOps if ops is None else ops
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        w, c, d = self.world, self.capacity, d_model
        self.header = int(self.ops.header_rows(self.experts_per_rank, c, d))
        bf = dict(dtype=torch.bfloat16, device=self.device)
        i32 = dict(dtype=torch.int32, device=self.device)
        if exchange not in ("nccl", "p2p"):
            raise ValueError(f"unknown exchange {exchange!r}")
        self.exchange = exchange
        self.peers = None
        self.ret_send = torch.zeros(w * c, d, **bf)
        if exchange == "p2p":
            # receive / return segments live in the IPC buffer the peers store into
            self.peers = PeerBuffers(w, self.rank, self.header + c, c, d, self.device, group)
            self.send = None
            self.recv, self.ret_recv = self.peers.recv, self.peers.ret_recv
            self.sync = torch.zeros(3, **i32)
        else:
            self.send = torch.zeros(w * (self.header + c), d, **bf)
            self.recv = torch.zeros_like(self.send)
            self.ret_recv = torch.zeros_like(self.ret_send)
        self.offsets_l = torch.zeros(self.experts_per_rank + 1, **i32)
        self.perm_token_l = torch.zeros(w * c, **i32)
        self.perm_prob_l = torch.zeros(w * c, dtype=torch.float32, device=self.device)
        self.out_row = torch.zeros(w * c, **i32)
        self.tile_offsets_l = torch.zeros(self.experts_per_rank + 1, **i32)
        self.tile_m = 128
        self.scratch = torch.zeros(int(self.ops.scratch_bytes(self)), dtype=torch.uint8,
                                   device=self.device)
        self.ret_route_pos = torch.zeros(c, **i32)

    @property
    def expert_range(self) -> tuple[int, int]:
        lo = self.rank * self.experts_per_rank
        return lo, lo + self.experts_per_rank

    def _exchange(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        dist.all_to_all_single(out, inp, group=self.group)

    def run(self, x: torch.Tensor, plan: kernels.RoutePlan, w13_local: torch.Tensor,
            w2_local: torch.Tensor, path: str = "auto") -> EpResult:
        """Routed expert outputs for this rank's routes.

        x [N, D] bf16 (the normalised MoE input), plan from kernels.route over
        all E experts (N*k <= capacity); w13_local [El, 2F, D] / w2_local
        [El, D, F] this rank's experts.  path: "grouped" (tcgen05 GEMMs),
        "decode" (weight streaming) or "auto", which picks from the capacity
        so that every rank makes the same choice (W*C rows over W*El experts,
        the single-device rule at a full batch).  Collective: every rank of
        the group must call it, in the same order.
        """
        n_routes = plan.perm_token.numel()
        if n_routes > self.capacity:
            raise ValueError(f"{n_routes} routes exceed the capacity {self.capacity}")
        if w13_local.shape[0] != self.experts_per_rank:
            raise ValueError("w13_local must hold this rank's experts only")
        rp = self.ret_route_pos[:n_routes]
        self.ops.dispatch_pack(self, x, plan, rp)
        if self.peers is None:
            self._exchange(self.recv, self.send)
        self.ops.recv_plan(self)
        if path not in ("auto", "grouped", "decode"):
            raise ValueError(f"unknown expert path {path!r}")
        grouped = path == "grouped" or (
            path == "auto" and kernels.use_grouped_rows(self.capacity, self.experts_per_rank,
                                                        self.d_model, self.ffn))
        self.ops.experts_to(self, w13_local, w2_local, grouped)
        if self.peers is None:
            self._exchange(self.ret_recv, self.ret_send)
        else:
            self.ops.return_push(self)
        return EpResult(self.ret_recv, rp)

    def check(self) -> None:
        """Raise if a device step of the exchange recorded an error in the device
        status word: a flag wait that ran out (a peer that never published,
        LLMYB_ETIMEOUT) or a malformed segment header (LLMYB_EINVAL).  Waits
        for the device.  LoopedHybridModel calls it after every eager forward
        and decode step; a caller replaying a captured step calls it at its
        own synchronisation points."""
        kernels.check_device_status(self.device)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (peer-memory exchange)."""
        if self.peers is not None:
            self.peers.close()
            self.peers = None
