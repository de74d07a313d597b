"""Expert-parallel exchange on CPU: world-size-2 gloo ranks drive the real
ExpertParallel host class with the numpy oracle steps injected, and the routed
outputs must equal a single-process computation of the same routes bit for bit.

This covers the host logic of the N>1 path (buffer sizing, segment layout,
exchange order, route remapping for the combine); the CUDA kernels of the same
steps are compared with the oracle in test_gpu_ep.py.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ep as oep
from oracle import routing


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).numpy().view(np.uint16)


def unpack_w13(w13_bits: np.ndarray):
    """Inverse of the 256-row gate/up interleave of llmyb_moe_pack_w13."""
    e, f2, d = w13_bits.shape
    t = w13_bits.reshape(e, f2 // 256, 2, 128, d)
    return t[:, :, 0].reshape(e, f2 // 2, d), t[:, :, 1].reshape(e, f2 // 2, d)


def pack_w13(gate_bits: np.ndarray, up_bits: np.ndarray) -> np.ndarray:
    e, f, d = gate_bits.shape
    g = gate_bits.reshape(e, f // 128, 1, 128, d)
    u = up_bits.reshape(e, f // 128, 1, 128, d)
    return np.concatenate([g, u], axis=2).reshape(e, 2 * f, d)


class OracleOps:
    """The device steps of ExpertParallel.run, restated by oracle/ep.py on CPU tensors."""

    header_rows = staticmethod(oep.header_rows)

    @staticmethod
    def scratch_bytes(ep) -> int:
        return 16

    @staticmethod
    def dispatch_pack(ep, x, plan, ret_route_pos):
        d, w, c = ep.d_model, ep.world, ep.capacity
        oep.dispatch_pack(_bits(x), plan.offsets.numpy(), plan.perm_token.numpy(),
                          plan.perm_prob.numpy(), plan.route_pos.numpy(), ep.n_experts, w, c,
                          _bits(ep.send).reshape(w, ep.header + c, d), ret_route_pos.numpy())

    @staticmethod
    def recv_plan(ep):
        d, w, c = ep.d_model, ep.world, ep.capacity
        off, pt, pp, orow = oep.recv_plan(_bits(ep.recv).reshape(w, ep.header + c, d), w, c,
                                          ep.experts_per_rank)
        ep.offsets_l.copy_(torch.from_numpy(off.astype(np.int32)))
        n = len(pt)
        ep.perm_token_l[:n] = torch.from_numpy(pt.astype(np.int32))
        ep.perm_prob_l[:n] = torch.from_numpy(pp)
        ep.out_row[:n] = torch.from_numpy(orow.astype(np.int32))

    @staticmethod
    def experts_to(ep, w13, w2, grouped):
        gate, up = unpack_w13(_bits(w13))
        n = int(ep.offsets_l[-1])
        oep.experts_to(_bits(ep.recv), ep.offsets_l.numpy(), ep.perm_token_l.numpy()[:n],
                       ep.perm_prob_l.numpy()[:n], ep.out_row.numpy()[:n], oep.bf16_value(gate),
                       oep.bf16_value(up), oep.bf16_value(_bits(w2)), _bits(ep.ret_send))


E, K, D, F = 8, 2, 64, 256


def _weights():
    rng = np.random.default_rng(7)
    gate = oep.bf16_bits(rng.normal(0, 0.1, (E, F, D)))
    up = oep.bf16_bits(rng.normal(0, 0.1, (E, F, D)))
    down = oep.bf16_bits(rng.normal(0, 0.1, (E, D, F)))
    return gate, up, down


def _tokens(rank: int, n: int, skew: bool):
    rng = np.random.default_rng(100 + rank)
    x = oep.bf16_bits(rng.normal(0, 1, (n, D)))
    logits = rng.normal(0, 1, (n, E)).astype(np.float32)
    if skew:  # every route lands on rank 0's experts: a full dispatch segment
        logits[:, : E // 2] += 100.0
    return x, logits


def _plan(logits: np.ndarray):
    from hybrid_llm_b200.kernels import RoutePlan
    idx, prob = routing.router_topk(logits, K)
    prob = prob.astype(np.float32)
    p = routing.dispatch_plan(idx, E)
    i32 = lambda a: torch.from_numpy(np.asarray(a, dtype=np.int32))
    return RoutePlan(
        topk_idx=torch.from_numpy(idx), topk_prob=torch.from_numpy(prob), counts=i32(p["counts"]),
        offsets=i32(p["offsets"]), tile_offsets=i32(p["tile_offsets"]),
        perm_token=i32(p["perm_token"]),
        perm_prob=torch.from_numpy(prob.reshape(-1)[p["sort_order"]].copy()),
        route_pos=i32(p["route_pos"]), sort_order=None), idx, prob


def _single_device(x_bits, idx, prob, gate, up, down):
    n = x_bits.shape[0]
    y = np.zeros((n * K, D), dtype=np.uint16)
    xv = oep.bf16_value(x_bits)
    for t in range(n):
        for s in range(K):
            e = idx[t, s]
            y[t * K + s] = oep.expert_rows(xv[t:t + 1], prob[t, s:s + 1], oep.bf16_value(gate[e]),
                                           oep.bf16_value(up[e]), oep.bf16_value(down[e]))[0]
    return oep.combine(y, np.arange(n * K), n, K)


def _worker(rank: int, world: int, port: int, n_tokens: list[int], skew: bool, max_tokens: int,
            errors):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from hybrid_llm_b200.expert_parallel import ExpertParallel
        gate, up, down = _weights()
        ep = ExpertParallel(E, K, D, F, max_tokens, device="cpu", ops=OracleOps)
        lo, hi = ep.expert_range
        w13 = torch.from_numpy(pack_w13(gate[lo:hi], up[lo:hi]).view(np.int16)).view(torch.bfloat16)
        w2 = torch.from_numpy(down[lo:hi].copy().view(np.int16)).view(torch.bfloat16)
        for step in range(2):  # buffers are reused across calls
            x_bits, logits = _tokens(rank + 10 * step, n_tokens[rank], skew)
            plan, idx, prob = _plan(logits)
            x = torch.from_numpy(x_bits.view(np.int16)).view(torch.bfloat16)
            res = ep.run(x, plan, w13, w2)
            got = oep.combine(_bits(res.y_rows), res.route_pos.numpy(), n_tokens[rank], K)
            want = _single_device(x_bits, idx, prob, gate, up, down)
            assert got.shape == want.shape
            assert np.array_equal(got, want), f"rank {rank} step {step}: EP != single device"
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:  # report to the parent, which fails the test
        errors.put(f"rank {rank}: {exc!r}")
        raise


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("n_tokens,skew", [([5, 7], False), ([6, 6], True), ([0, 4], False)])
def test_ep_exchange_matches_single_device(n_tokens, skew):
    ctx = mp.get_context("spawn")
    errors = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(2, _free_port(), n_tokens, skew, max(n_tokens), errors),
                       nprocs=2, join=True, start_method="spawn")
    assert errors.empty(), errors.get()


def test_recv_plan_order():
    """Rows of one local expert are ordered by source rank, then source order."""
    world, cap, el, d = 2, 4, 2, 8
    h = oep.header_rows(el, cap, d)
    recv = np.zeros((world, h + cap, d), dtype=np.uint16)
    # rank 0 sent 1 row for expert 0 and 2 for expert 1; rank 1 sent 2 for expert 0
    for p, counts in enumerate([[1, 2], [2, 0]]):
        hdr = recv[p, :h].reshape(-1).view(np.int32)
        hdr[:el] = counts
        hdr.view(np.float32)[el:el + sum(counts)] = np.arange(sum(counts)) + 10 * p
    off, pt, pp, orow = oep.recv_plan(recv, world, cap, el)
    assert off.tolist() == [0, 3, 5]
    assert orow.tolist() == [0, 4, 5, 1, 2]          # e0: (0,0) (1,0) (1,1); e1: (0,1) (0,2)
    assert pt.tolist() == [h, h + cap + h, h + cap + h + 1, h + 1, h + 2]
    assert pp.tolist() == [0.0, 10.0, 11.0, 1.0, 2.0]
