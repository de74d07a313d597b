"""Expert-parallel kernels (csrc/ep.cu, llmyb_moe_decode_experts_to) on the GPU.

* One GPU, W emulated ranks: dispatch_pack / recv_plan / experts_to run per
  rank; the all-to-all is done with segment copies.  Every packed segment and
  plan must equal oracle/ep.py bit for bit, and the combined output must
  equal the single-device path (route + moe_decode_experts + routed add)
  bit for bit.
* Two or more GPUs: the same through ExpertParallel with NCCL, one process
  per GPU (skipped when fewer GPUs are visible).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from oracle import ep as oep

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _setup(dev, world, e, k, d, f, n_per_rank, seed=0, skew=False):
    from hybrid_llm_b200 import kernels
    g = torch.Generator(device="cpu").manual_seed(seed)
    wg = (torch.randn(e, f, d, generator=g) * 0.05).bfloat16().to(dev)
    wu = (torch.randn(e, f, d, generator=g) * 0.05).bfloat16().to(dev)
    wd = (torch.randn(e, d, f, generator=g) * 0.05).bfloat16().to(dev)
    w13 = kernels.pack_w13(wg, wu)
    xs, plans = [], []
    for r in range(world):
        x = torch.randn(n_per_rank[r], d, generator=g).bfloat16().to(dev)
        logits = torch.randn(n_per_rank[r], e, generator=g)
        if skew:
            logits[:, : e // world] += 50.0
        plans.append(kernels.route(logits.to(dev), k, tile_m=128))
        xs.append(x)
    return w13, wd, xs, plans


def _single_device(x, plan, w13, wd, d, grouped=False):
    from hybrid_llm_b200 import kernels
    if grouped:
        n = plan.perm_token.numel()
        y = torch.empty(n, d, dtype=torch.bfloat16, device=x.device)
        scratch = torch.empty(kernels.grouped_scratch_bytes(n, d, wd.shape[-1]), dtype=torch.uint8,
                              device=x.device)
        kernels.moe_grouped_experts_to(x, n, plan.perm_token, plan.perm_prob, plan.offsets,
                                       plan.tile_offsets, 128, w13, wd, scratch, y)
    else:
        y = kernels.moe_decode_experts(x, plan, w13, wd)
    streams = torch.zeros(x.shape[0], d, dtype=torch.float32, device=x.device)
    kernels.add_rmsnorm_routed(streams, y, plan, None, 1e-6, normalize=False)
    return streams


@pytest.mark.parametrize("grouped", [False, True])
@pytest.mark.parametrize("world,e,k,d,f,n,skew", [
    (2, 8, 2, 256, 256, [5, 9], False),
    (4, 16, 4, 512, 384, [7, 1, 0, 12], False),
    (4, 16, 4, 256, 256, [6, 6, 6, 6], True),
    (8, 64, 8, 2048, 1024, [8] * 8, False),     # the large expert-parallel config's shapes
])
def test_ep_kernels_emulated_ranks(cuda, world, e, k, d, f, n, skew, grouped):
    from hybrid_llm_b200 import kernels
    from dataclasses import replace
    w13, wd, xs, plans = _setup(cuda, world, e, k, d, f, n, skew=skew)
    el = e // world
    cap = max(n) * k
    h = kernels.ep_header_rows(el, cap, d)
    assert h == oep.header_rows(el, cap, d)
    sends, rps = [], []
    for r in range(world):
        send = torch.zeros(world * (h + cap), d, dtype=torch.bfloat16, device=cuda)
        rp = torch.full((max(cap, 1),), -1, dtype=torch.int32, device=cuda)
        kernels.ep_dispatch_pack(xs[r], plans[r], e, world, cap, send, rp)
        # oracle on the same plan
        p = plans[r]
        want = np.zeros((world, h + cap, d), dtype=np.uint16)
        want_rp = np.zeros(p.perm_token.numel(), dtype=np.int32)
        oep.dispatch_pack(_bits(xs[r]), p.offsets.cpu().numpy(), p.perm_token.cpu().numpy(),
                          p.perm_prob.cpu().numpy(), p.route_pos.cpu().numpy(), e, world, cap,
                          want, want_rp)
        got = _bits(send).reshape(world, h + cap, d)
        counts = np.diff(p.offsets.cpu().numpy())
        for q in range(world):
            c = int(counts[q * el:(q + 1) * el].sum())
            hdr_g = got[q, :h].reshape(-1).view(np.int32)
            hdr_w = want[q, :h].reshape(-1).view(np.int32)
            assert np.array_equal(hdr_g[:el + c], hdr_w[:el + c])
            assert np.array_equal(got[q, h:h + c], want[q, h:h + c])
        n_routes = p.perm_token.numel()
        assert np.array_equal(rp[:n_routes].cpu().numpy(), want_rp)
        sends.append(send.view(world, h + cap, d))
        rps.append(rp[:n_routes])
    # all-to-all by copies: recv_q[p] = send_p[q]
    recvs = [torch.stack([sends[p][q] for p in range(world)]).reshape(-1, d) for q in range(world)]
    rets = []
    for q in range(world):
        off = torch.zeros(el + 1, dtype=torch.int32, device=cuda)
        pt = torch.zeros(world * cap, dtype=torch.int32, device=cuda)
        pp = torch.zeros(world * cap, dtype=torch.float32, device=cuda)
        orow = torch.zeros(world * cap, dtype=torch.int32, device=cuda)
        toff = torch.zeros(el + 1, dtype=torch.int32, device=cuda)
        kernels.ep_recv_plan(recvs[q], world, cap, el, off, pt, pp, orow, tile_offsets_l=toff,
                             tile_m=128)
        w_off, w_pt, w_pp, w_or = oep.recv_plan(_bits(recvs[q]).reshape(world, h + cap, d), world,
                                                cap, el)
        m = int(w_off[-1])
        assert off.cpu().numpy().tolist() == w_off.tolist()
        assert pt[:m].cpu().numpy().tolist() == w_pt.tolist()
        assert np.array_equal(pp[:m].cpu().numpy(), w_pp)
        assert orow[:m].cpu().numpy().tolist() == w_or.tolist()
        cnt = np.diff(w_off)
        assert toff.cpu().numpy().tolist() == np.concatenate([[0], np.cumsum((cnt + 127) // 128)]).tolist()
        ret = torch.zeros(world * cap, d, dtype=torch.bfloat16, device=cuda)
        we13, we2 = w13[q * el:(q + 1) * el], wd[q * el:(q + 1) * el]
        if grouped:
            scratch = torch.empty(kernels.grouped_scratch_bytes(world * cap, d, f),
                                  dtype=torch.uint8, device=cuda)
            kernels.moe_grouped_experts_to(recvs[q], world * cap, pt, pp, off, toff, 128, we13,
                                           we2, scratch, ret, orow)
        else:
            hs = torch.zeros(world * cap, f, dtype=torch.bfloat16, device=cuda)
            kernels.moe_decode_experts_to(recvs[q], world * cap, pt, pp, off, we13, we2, hs, ret,
                                          orow)
        rets.append(ret.view(world, cap, d))
    for r in range(world):
        if n[r] == 0:
            continue
        ret_recv = torch.stack([rets[q][r] for q in range(world)]).reshape(-1, d)
        streams = torch.zeros(n[r], d, dtype=torch.float32, device=cuda)
        kernels.add_rmsnorm_routed(streams, ret_recv, replace(plans[r], route_pos=rps[r]), None,
                                   1e-6, normalize=False)
        want = _single_device(xs[r], plans[r], w13, wd, d, grouped)
        assert torch.equal(streams, want), f"rank {r}: expert-parallel != single device"


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, errors):
    import torch.distributed as dist
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        from datetime import timedelta
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=timedelta(seconds=60))
        from hybrid_llm_b200.expert_parallel import ExpertParallel
        e, k, d, f = 16, 4, 512, 256
        n = [3 + 2 * r for r in range(world)]
        w13, wd, xs, plans = _setup(dev, world, e, k, d, f, n, seed=3)
        from hybrid_llm_b200 import kernels
        for exchange in ("nccl", "p2p"):
            ep = ExpertParallel(e, k, d, f, max(n), device=dev, exchange=exchange)
            lo, hi = ep.expert_range
            for path in ("decode", "grouped", "decode"):
                res = ep.run(xs[rank], plans[rank], w13[lo:hi].contiguous(),
                             wd[lo:hi].contiguous(), path=path)
                streams = torch.zeros(n[rank], d, dtype=torch.float32, device=dev)
                kernels.add_rmsnorm_routed(streams, res.y_rows, res.plan_for_combine(plans[rank]),
                                           None, 1e-6, normalize=False)
                want = _single_device(xs[rank], plans[rank], w13, wd, d, grouped=path == "grouped")
                assert torch.equal(streams, want), \
                    f"rank {rank}: {exchange} expert-parallel != single device"
            torch.cuda.synchronize()
            kernels.check_device_status()
            dist.barrier()
            ep.close()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:
        errors.put(f"rank {rank}: {exc!r}")
        raise


def test_ep_nccl_two_or_more_gpus(cuda):
    import torch.multiprocessing as mp
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs two or more GPUs")
    world = min(world, 4)
    ctx = mp.get_context("spawn")
    errors = ctx.SimpleQueue()
    mp.start_processes(_nccl_worker, args=(world, _free_port(), errors), nprocs=world, join=True,
                       start_method="spawn")
    assert errors.empty(), errors.get()


def _model_worker(rank, world, port, errors):
    import torch.distributed as dist
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        from datetime import timedelta
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=timedelta(seconds=60))
        from hybrid_llm_b200.config import HybridConfig
        from hybrid_llm_b200.expert_parallel import ExpertParallel
        from hybrid_llm_b200.model import LoopedHybridModel
        from hybrid_llm_b200.state import RecurrentState
        from hybrid_llm_b200.weights import ModelWeights, synthetic_state_dict
        cfg = HybridConfig(vocab_size=512, d_model=256, recurrent_layout=("csa_moe", "gdn_moe") * 2,
                           num_loops=2, gdn_heads=2, gdn_key_dim=64, gdn_value_dim=64, csa_heads=4,
                           csa_head_dim=64, csa_window=16, moe_experts=8, moe_top_k=2,
                           moe_hidden=256, name="ep-test")
        bsz, t = 2, 24
        sd = synthetic_state_dict(cfg, seed=5, device=dev, std=0.05)
        full = LoopedHybridModel(ModelWeights.from_state_dict(cfg, sd, dev))
        ep = ExpertParallel(cfg.moe_experts, cfg.moe_top_k, cfg.d_model, cfg.moe_hidden, bsz * t,
                            device=dev, exchange="p2p")
        shard = LoopedHybridModel(ModelWeights.from_state_dict(cfg, sd, dev,
                                                               expert_range=ep.expert_range), ep=ep)
        g = torch.Generator(device="cpu").manual_seed(100 + rank)
        ids = torch.randint(0, cfg.vocab_size, (bsz, t), generator=g).to(dev)
        # with the same expert kernels on both sides the expert-parallel rows are
        # bit-identical to the single-device ones, and so are prefill and decode
        for path in ("decode", "grouped"):
            full.expert_path = shard.expert_path = path
            out_full = full.forward(ids, last_logits_only=True)
            out_ep = shard.forward(ids, last_logits_only=True)
            assert torch.equal(out_full.logits, out_ep.logits), \
                f"rank {rank}: {path} expert-parallel prefill differs"
            a = out_full.logits.float()
            st_full = RecurrentState(cfg, bsz, dev)
            st_full.load_state_dict(out_full.state.state_dict())
            st_ep = RecurrentState(cfg, bsz, dev)
            st_ep.load_state_dict(out_ep.state.state_dict())
            tok = a[:, -1].argmax(-1)
            for _ in range(4):
                la = full.decode_step(tok, st_full)
                lb = shard.decode_step(tok, st_ep)
                assert torch.equal(la, lb), f"rank {rank}: {path} expert-parallel decode differs"
                tok = la.float().argmax(-1)
        shard.expert_path = "auto"
        # the peer-memory exchange inside a captured CUDA graph
        from hybrid_llm_b200.model import GreedyDecoder
        toks = []
        for use_graph in (False, True):
            st = RecurrentState(cfg, bsz, dev)
            st.load_state_dict(out_full.state.state_dict())
            dec = GreedyDecoder(shard, st, use_graph=use_graph)
            dec.prime(a[:, -1].argmax(-1))
            toks.append(torch.stack([dec.step().clone() for _ in range(4)], 1))
            del dec
        assert torch.equal(toks[0], toks[1]), f"rank {rank}: graph decode differs"
        torch.cuda.synchronize()
        from hybrid_llm_b200 import kernels
        kernels.check_device_status()
        dist.barrier()
        ep.close()
        dist.destroy_process_group()
    except BaseException as exc:
        errors.put(f"rank {rank}: {exc!r}")
        raise


def test_ep_model_decode_two_or_more_gpus(cuda):
    import torch.multiprocessing as mp
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs two or more GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    errors = ctx.SimpleQueue()
    mp.start_processes(_model_worker, args=(world, _free_port(), errors), nprocs=world, join=True,
                       start_method="spawn")
    assert errors.empty(), errors.get()
