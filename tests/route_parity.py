"""Routing-aware model parity (GPU model against the CPU oracle).

The random-init test models route on nearly flat router logits, so a bf16
path resolves some near ties between the k-th and (k+1)-th expert the other
way than the fp64 oracle, and one flipped expert moves a token's logits far
beyond any bf16 tolerance.  The comparison therefore:

1. records the experts the GPU chose in every MoE call (model.route_log);
2. runs the oracle with those experts forced (oracle.model.OracleModel
   forced_routes; probabilities still from its own logits) and requires
   every GPU choice that differs from the oracle's own top-k to be a near
   tie: each chosen expert's oracle logit within `tie` of the row's logit
   range below the oracle's k-th largest logit;
3. compares the GPU logits with the forced oracle within `logit_rel` of
   max |ref|, and with the reference's golden logits as well wherever no
   routing decision differed.
"""
from __future__ import annotations

import numpy as np
import torch


def rel(a, b) -> float:
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def route_mismatches(oracle_log, gpu_routes, tie: float):
    """(mismatches, worst near-tie gap); asserts every mismatch is a near tie."""
    assert len(oracle_log) == len(gpu_routes), (len(oracle_log), len(gpu_routes))
    mism, worst = 0, 0.0
    for (own, lg), got in zip(oracle_log, gpu_routes):
        got = np.asarray(got, np.int64).reshape(own.shape)
        k = own.shape[1]
        lg = np.asarray(lg, np.float64).reshape(own.shape[0], -1)
        kth = -np.sort(-lg, -1)[:, k - 1]
        span = lg.max(-1) - lg.min(-1)
        gap = (kth - np.take_along_axis(lg, got, -1).min(-1)) / span
        diff = (np.sort(own, -1) != np.sort(got, -1)).any(-1)
        mism += int(diff.sum())
        if diff.any():
            worst = max(worst, float(gap[diff].max()))
    assert worst <= tie, f"a routing mismatch {worst:.3e} of the logit range away from a tie"
    return mism, worst


def _forced(orc, routes, fn, *args):
    orc.forced_routes = [np.asarray(r) for r in routes]
    orc.route_log = []
    out = fn(*args)
    assert not orc.forced_routes, "the oracle made fewer MoE calls than the GPU"
    log, orc.route_log, orc.forced_routes = orc.route_log, None, None
    return out, log


def check_model(model, orc, ids: np.ndarray, tokens: np.ndarray, golden_prefill=None,
                golden_steps=None, logit_rel: float = 3e-2, tie: float = 2e-2) -> dict:
    """Prefill of ids [B, T], then one decode step per column of tokens [B, S]
    (teacher forced), on the GPU model and on the oracle with the GPU's
    routes.  golden_prefill [B, V] / golden_steps [B, S, V]: the reference's
    own logits, compared wherever routing agreed.  Returns statistics."""
    from hybrid_llm_b200 import kernels
    stats = dict(mismatches=0, worst_tie=0.0, worst_rel=0.0, golden_compared=0)

    def step_check(tag, got, log, routes, ref, gold):
        mism, worst = route_mismatches(log, routes, tie)
        stats["mismatches"] += mism
        stats["worst_tie"] = max(stats["worst_tie"], worst)
        e = rel(got, ref)
        stats["worst_rel"] = max(stats["worst_rel"], e)
        assert e < logit_rel, f"{tag}: logits {e:.3e} of max |ref| off the routing-forced oracle"
        if gold is not None and mism == 0:
            g = rel(got, gold)
            assert g < logit_rel, f"{tag}: logits {g:.3e} of max |ref| off the reference"
            stats["golden_compared"] += 1

    model.route_log = []
    out = model.forward(torch.from_numpy(ids).cuda(), last_logits_only=True)
    got = out.logits[:, -1].float().cpu().numpy()
    routes = [r.cpu().numpy() for r in model.route_log]
    (ref, st), log = _forced(orc, routes, orc.forward, ids)
    step_check("prefill", got, log, routes, ref[:, -1], golden_prefill)
    state = out.state
    for i in range(tokens.shape[1]):
        model.route_log = []
        got = model.decode_step(torch.from_numpy(tokens[:, i]).cuda(), state).float().cpu().numpy()
        routes = [r.cpu().numpy() for r in model.route_log]
        (ref_s, st), log = _forced(orc, routes, orc.decode_step, tokens[:, i], st)
        step_check(f"step {i}", got, log, routes, ref_s,
                   None if golden_steps is None else golden_steps[:, i])
    model.route_log = None
    kernels.check_device_status()
    return stats
