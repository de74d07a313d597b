"""Benchmark of the B200-native looped hybrid LLMY stack (one JSON line on rank 0).

Headline workload (N=1): the full small LLMY model (vocab 32000, d_model 768,
12 alternating CSA/GDN blocks with a 16-expert top-2 MoE in each, 2 loops),
bf16, random-init N(0, 0.02) weights, a 512-token prompt of uniform ids,
then greedy decode at batch 1.  One step = one decoded token: the whole
decode step (embedding -> 2 x 12 blocks -> LM head -> sampler) is one CUDA
graph replay, the sampled token feeding the next step on the device.

  value   decode tokens/s with everything resident on the device
  e2e     the same through the public decode API with a pinned-host token
          round trip every step (H2D of the input id, D2H of the sampled id
          and its log-probability)
  secondary  the single looped block ([1, 256, 512], 2 loops), isolated-MoE-
          layer TFLOPS (16384 tokens x 1024, 32 experts top-4, Zipf-skewed
          routing), long-context prefill (banded attention and the GDN chunked
          scan at B=8, T=8192), the large expert-parallel decode (batch 64),
          small-model prefill tokens/s
  cpu_baseline  the CPU port of the reference algorithm (oracle/) timed on
          this host on a bounded sample of the same decode workload

Under torchrun (N > 1) every rank decodes its own replica (the decode path
has no cross-GPU exchange: "replicas only"), the time is the max over ranks
and value is the sum of all ranks' tokens / that time.

``--impl reference`` times the CPU port of the reference's decode path on the
host cores (rank 0 only), with the same metric and workload.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s (B=1, B=64), prefill tok/s, MoE TFLOPS at 1/2/4/8 B200"
WORKLOAD = "small-llmy greedy decode B=1 (vocab 32000, d768, 12 blocks csa/gdn+moe16top2, 2 loops, prompt 512)"


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        import statistics
        rows = []
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                    rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, val in zip(names, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]),
                "reasons": sorted(reasons), "samples": len(rows)}


# ------------------------------------------------------------ CPU baseline
def cpu_decode_baseline(steps: int, warmup: int, prompt_len: int = 16,
                        budget_s: float | None = None) -> dict:
    """Time the CPU port of the reference decode path (oracle/) on this host.

    Same model shape as the GPU workload, fp32 numpy, batch 1.  The prompt is
    shortened to bound the (untimed) prefill; per-token decode work differs
    only in the CSA window length (negligible next to the dense and expert
    GEMVs).  Weights are N(0, 0.02) from numpy's generator (values do not
    affect the timing).
    """
    import numpy as np
    import torch

    from hybrid_llm_b200.config import small_llmy_config
    from hybrid_llm_b200.weights import parameter_shapes
    from oracle.model import OracleModel

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    cfg = small_llmy_config()
    rng = np.random.default_rng(0)
    sd = {}
    for name, shape in parameter_shapes(cfg).items():
        if len(shape) >= 2:
            sd[name] = rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)
        elif name.endswith("decay_logit"):
            sd[name] = np.full(shape, 2.0, np.float32)
        elif name.endswith("beta_proj.bias"):
            sd[name] = np.zeros(shape, np.float32)
        else:
            sd[name] = np.ones(shape, np.float32)
    m = OracleModel(cfg, sd, dtype=np.float32)
    ids = rng.integers(0, cfg.vocab_size, (1, prompt_len))
    logits, st = m.forward(ids)
    tok = logits[:, -1].argmax(-1)
    tw = time.perf_counter()
    for _ in range(warmup):
        logits, st = m.decode_step(tok, st)
        tok = logits.argmax(-1)
    capped = False
    if budget_s is not None and warmup > 0:
        per_token = (time.perf_counter() - tw) / warmup
        limit = max(1, int(budget_s / max(per_token, 1e-9)))
        capped, steps = steps > limit, min(steps, limit)
    t0 = time.perf_counter()
    for _ in range(steps):
        logits, st = m.decode_step(tok, st)
        tok = logits.argmax(-1)
    dt = time.perf_counter() - t0
    res = {"value": steps / dt, "unit": "tok/s", "cores": cores, "kind": "port", "steps": steps,
           "sample": f"{steps} greedy decode tokens at B=1 after a {prompt_len}-token prompt, "
                     f"fp32 numpy port of the reference decode path, {cores} host threads"}
    if capped:
        res["note"] = f"timed tokens capped at {steps} to keep the run within {budget_s:.0f} s"
    return res


# -------------------------------------------------------------- reference
def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # one step = one greedy decode token of the CPU port; K steps after W
    # warm-up tokens, K capped (and reported) if the run would exceed ~2.5 min
    res = cpu_decode_baseline(steps=max(1, args.steps), warmup=args.warmup, budget_s=150.0)
    steps = res.pop("steps")
    line = {
        "impl": "reference", "metric": METRIC, "value": res["value"], "unit": "tok/s",
        "n_gpus": args.gpus, "steps": steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": WORKLOAD + " [CPU port, prompt 16]"},
        "cpu_baseline": res,
        "e2e": {"value": res["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- our path
# DRAM traffic of one decode_out_router_cluster_kernel launch at the small-llmy
# decode shape, measured with ncu (dram__bytes_read.sum + dram__bytes_write.sum,
# caches flushed before the launch; two launches: 1,305,344 and 1,323,520 bytes).
OUT_ROUTER_TRAFFIC = 1_314_432
# ncu dram__bytes_read.sum + dram__bytes_write.sum of one decode_persistent_kernel
# launch at the benchmark's decode shape (small LLMY, 512-token prompt, sixth
# decode step): 412,692,992 read + 5,650,944 written
PERSISTENT_TRAFFIC = 418_343_936


def out_router_roofline(model, p: dict, reps: int = 50) -> dict:
    """Roofline of the decode step's dominant kernel (decode_out_router_cluster_kernel:
    output projection + residual + norms + router of one block, the largest
    share of the step's launch list) at the benchmark's decode shape.  Its
    average launch duration is timed with CUDA events over a CUDA graph of
    `reps` launches on the stream it runs on; the inputs are scratch copies,
    so the decode state is untouched."""
    import torch

    from hybrid_llm_b200 import kernels
    from hybrid_llm_b200.weights import CsaBlock

    cfg = model.cfg
    d = cfg.d_model
    blk = next(b for b in model.w.blocks if isinstance(b.mixer, CsaBlock))
    g = torch.Generator(device="cuda").manual_seed(3)
    inp = torch.randn(1, d, device="cuda", generator=g).bfloat16()
    streams = torch.randn(1, d, device="cuda", generator=g)
    m_bf = torch.empty(1, d, dtype=torch.bfloat16, device="cuda")
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    call = lambda: kernels.decode_out_router(inp, blk.mixer.w_o, streams, blk.ffn_norm,
                                             blk.moe.router_folded, cfg.moe_top_k, cfg.rms_eps,
                                             m_bf, counter, tile_m=128)
    call()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        call()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(reps):
            call()
    graph.replay()
    torch.cuda.synchronize()
    a, b = _events()
    a.record()
    for _ in range(5):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    dt = a.elapsed_time(b) * 1e-3 / (5 * reps)
    nb = lambda t: t.numel() * t.element_size()
    alg = (nb(blk.mixer.w_o) + nb(blk.moe.router_folded) + nb(blk.ffn_norm) + nb(inp)
           + 2 * nb(streams) + nb(m_bf))
    achieved = alg / dt / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": p["hbm_gbs"], "unit": "GB/s",
            "frac": achieved / p["hbm_gbs"], "traffic": OUT_ROUTER_TRAFFIC,
            "kernel": "decode_out_router_cluster_kernel (CSA block, batch 1): one 8-CTA cluster; "
                      "output projection GEMV + residual + norm and router-logit shares per CTA, "
                      "combined through distributed shared memory; top-k/plan in CTA 0",
            "algorithmic_bytes_per_launch": alg, "avg_launch_us": dt * 1e6,
            "timing": f"CUDA events over a graph of {reps} launches x 5 replays",
            "peak_source": p["source"]}


def persistent_roofline(model, state, p: dict, reps: int = 20) -> dict:
    """Roofline of the decode step's kernel when the step is one persistent
    launch (llmyb_decode_persistent): algorithmic bytes per launch (every
    weight, cache and state byte the step touches, decode_bytes_per_step with
    the folded CSA projection) over the average launch time, timed with CUDA
    events over a CUDA graph of `reps` launches (each a 4-byte barrier reset +
    the kernel) on the stream they run on.  The launches advance a copy of the
    decode state."""
    import ctypes

    import torch

    from hybrid_llm_b200 import _native
    from hybrid_llm_b200.state import RecurrentState

    st = RecurrentState(model.cfg, state.batch, "cuda")
    st.load_state_dict(state.state_dict())
    pd = model._persistent_for(st)
    pd.prepare()
    lib = _native.lib()
    call = lambda: _native.check(lib.llmyb_decode_persistent(
        ctypes.byref(pd.params), torch.cuda.current_stream().cuda_stream), "persistent")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        call()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(reps):
            call()
    graph.replay()
    torch.cuda.synchronize()
    a, b = _events()
    a.record()
    for _ in range(3):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    dt = a.elapsed_time(b) * 1e-3 / (3 * reps)
    alg = decode_bytes_per_step(model, model.cfg, folded=True)
    achieved = alg / dt / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": p["hbm_gbs"], "unit": "GB/s",
            "frac": achieved / p["hbm_gbs"], "traffic": PERSISTENT_TRAFFIC,
            "kernel": "decode_persistent_kernel<3,4>: the whole batch-1 decode step (24 block "
                      "applications + collapse + final norm + LM head) as one cooperative "
                      "launch of one 512-thread CTA per SM, phases separated by grid barriers",
            "algorithmic_bytes_per_launch": alg, "avg_launch_us": dt * 1e6,
            "timing": f"CUDA events over a graph of {reps} launches x 3 replays",
            "peak_source": p["source"]}


def _events():
    import torch
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def secondary_block(p: dict, reps: int = 20) -> dict:
    """Single looped hybrid block workload: hidden states [1, 256, 512] ~ N(0, 1)
    through the csa_moe + gdn_moe core, 2 loops (random N(0, 0.02) weights).
    The reference runs it in fp32 on the CPU; here bf16 operands with fp32
    accumulation and an fp32 residual stream."""
    import numpy as np
    import torch

    from hybrid_llm_b200.config import single_block_config
    from hybrid_llm_b200.model import LoopedHybridModel, StackGraph
    from hybrid_llm_b200.weights import ModelWeights, synthetic_state_dict

    cfg = single_block_config()
    model = LoopedHybridModel(ModelWeights.from_state_dict(
        cfg, synthetic_state_dict(cfg, seed=0, device="cuda"), "cuda"))
    x = torch.from_numpy(np.random.default_rng(1).normal(0, 1, (1, 256, cfg.d_model))
                         .astype(np.float32)).cuda()

    def timed(fn):
        for _ in range(3):
            fn()
        times = []
        for _ in range(max(1, reps)):
            a, b = _events()
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b))
        return float(np.median(times)) * 1e-3

    t_eager = timed(lambda: model.run_stack(x))
    eager_out = model.run_stack(x)
    sg = StackGraph(model, 1, 256)
    t = timed(lambda: sg.run(x))
    same = bool(torch.equal(sg.run(x), eager_out))
    # MoE 2*T*k*3*D*F per block application (the dominant term), 2 blocks x 2 loops
    flops = 4 * 2.0 * 256 * cfg.moe_top_k * 3 * cfg.d_model * cfg.moe_hidden
    return {"workload": "single looped block [1, 256, 512], csa_moe + gdn_moe, 2 loops, "
                        "one CUDA graph replay (StackGraph)",
            "ms": t * 1e3, "tok_s": 256 / t, "moe_tflops": flops / t / 1e12,
            "eager_ms": t_eager * 1e3, "graph_equals_eager": same,
            "precision": "bf16 operands, fp32 accumulation and residual: measured against the "
                         "reference's fp32 configuration at the bf16 tolerance (2e-2 of the "
                         "residual update), not an fp32 result",
            "note": "latency-bound (256 tokens); timed with CUDA events, median; the eager "
                    "call (host launch cost included) in eager_ms"}


def secondary_moe(p: dict, reps: int = 10) -> dict:
    """Isolated MoE layer: 16384 x 1024 bf16, 32 experts top-4, F=512, Zipf bias."""
    import numpy as np
    import torch

    from hybrid_llm_b200 import kernels
    from oracle.routing import zipf_expert_bias

    n, d, e, k, f = 16384, 1024, 32, 4, 512
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(n, d, device="cuda", generator=g).bfloat16()
    wr = torch.randn(e, d, device="cuda", generator=g) * 0.02
    bias = torch.from_numpy(zipf_expert_bias(e)).cuda()
    wg = (torch.randn(e, f, d, device="cuda", generator=g) * 0.02).bfloat16()
    wu = (torch.randn(e, f, d, device="cuda", generator=g) * 0.02).bfloat16()
    wd = (torch.randn(e, d, f, device="cuda", generator=g) * 0.02).bfloat16()
    w13 = kernels.pack_w13(wg, wu)
    out = torch.empty(n, d, device="cuda", dtype=torch.bfloat16)
    scratch = torch.empty(int(kernels._native.lib().llmyb_moe_grouped_scratch_bytes(n, k, d, f)),
                          dtype=torch.uint8, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def layer():
        logits = torch.mm(x.float(), wr.t())
        plan = kernels.route(logits, k, bias)
        kernels.moe_grouped(x, plan, w13, wd, out=out, scratch=scratch)
        return plan

    for _ in range(3):
        plan = layer()
    times = []
    for _ in range(max(1, reps)):
        flush.zero_()
        a, b = _events()
        a.record()
        layer()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    t = float(np.median(times)) * 1e-3
    flops = 2.0 * n * k * 3 * f * d
    counts = plan.counts.cpu().tolist()
    # the routed experts alone (same plan): gather + the two tcgen05 grouped GEMMs
    rows = n * k
    y_rows = torch.empty(rows, d, device="cuda", dtype=torch.bfloat16)
    escratch = torch.empty(kernels.grouped_scratch_bytes(rows, d, f), dtype=torch.uint8,
                           device="cuda")
    experts = lambda: kernels.moe_grouped_experts_to(
        x, rows, plan.perm_token, plan.perm_prob, plan.offsets, plan.tile_offsets, plan.tile_m,
        w13, wd, escratch, y_rows)
    for _ in range(3):
        experts()
    etimes = []
    for _ in range(max(1, reps)):
        flush.zero_()
        a, b = _events()
        a.record()
        experts()
        b.record()
        torch.cuda.synchronize()
        etimes.append(a.elapsed_time(b))
    te = float(np.median(etimes)) * 1e-3
    return {"workload": "isolated MoE layer 16384x1024, 32 experts top-4, F=512, Zipf(1.1) bias",
            "ms": t * 1e3, "tflops": flops / t / 1e12,
            "frac_of_bf16_peak": flops / t / 1e12 / p["bf16_tflops"],
            "includes": "router logits GEMM + top-k/plan + gather + 2 grouped GEMMs + combine",
            "experts_ms": te * 1e3, "experts_tflops": flops / te / 1e12,
            "experts_frac_of_bf16_peak": flops / te / 1e12 / p["bf16_tflops"],
            "experts_includes": "row gather + GEMM1 (SwiGLU epilogue) + GEMM2 (probability "
                                "epilogue), L2 flushed before each call",
            "expert_load": counts}


def secondary_sampling_router(p: dict, reps: int = 20) -> dict:
    """The device sampler on a [64, 32000] fp32 logits block (temperature 0.8,
    top-k 50, top-p 0.9, repetition penalty 1.1 over a seen mask: the
    sample_standalone.py:5383-5423 path) and the router top-k + dispatch plan
    of the isolated MoE layer's shape (16,384 tokens x 32 experts, top-4,
    Zipf(1.1) bias), each timed alone with CUDA events (median), L2 flushed
    before every call; algorithmic bytes are the logits read plus what the
    kernels must write."""
    import numpy as np
    import torch

    from hybrid_llm_b200 import kernels
    from oracle.routing import zipf_expert_bias

    g = torch.Generator(device="cuda").manual_seed(0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def timed(fn):
        for _ in range(3):
            fn()
        ts = []
        for _ in range(max(1, reps)):
            flush.zero_()
            a, b = _events()
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        return float(np.median(ts)) * 1e-3

    bsz, vocab = 64, 32000
    logits = torch.randn(bsz, vocab, device="cuda", generator=g) * 3
    seen = torch.zeros(bsz, (vocab + 31) // 32, dtype=torch.int32, device="cuda")
    seen[:, :40].random_(generator=g)
    uni = torch.rand(bsz, device="cuda", generator=g)
    tok = torch.empty(bsz, dtype=torch.int64, device="cuda")
    lp = torch.empty(bsz, dtype=torch.float32, device="cuda")
    t_s = timed(lambda: kernels.sample(logits, temperature=0.8, top_k=50, top_p=0.9,
                                       repetition_penalty=1.1, seen=seen, uniforms=uni, out=tok,
                                       logprob=lp))
    s_bytes = bsz * vocab * 4 + seen.numel() * 4 + bsz * 12

    n, e, k = 16384, 32, 4
    rl = torch.randn(n, e, device="cuda", generator=g) * 0.5
    bias = torch.from_numpy(zipf_expert_bias(e)).cuda()
    t_r = timed(lambda: kernels.route(rl, k, bias))
    # logits read; top-k ids (8 B) + probs, the permutation's token, prob and
    # route position (4 B each) written per route; counts / offsets negligible
    r_bytes = n * e * 4 + n * k * (8 + 4) + n * k * (4 + 4 + 4)
    return {"workload": "sampler [64, 32000] fp32 (T 0.8, top-k 50, top-p 0.9, rep 1.1); "
                        "router top-k + plan 16384 x 32 top-4 (Zipf bias)",
            "sample_us": t_s * 1e6, "sample_gbs": s_bytes / t_s / 1e9,
            "sample_frac_of_hbm": s_bytes / t_s / 1e9 / p["hbm_gbs"],
            "route_us": t_r * 1e6, "route_gbs": r_bytes / t_r / 1e9,
            "route_frac_of_hbm": r_bytes / t_r / 1e9 / p["hbm_gbs"],
            "algorithmic_bytes": {"sample": s_bytes, "route": r_bytes}}


def secondary_prefill_c2(p: dict, reps: int = 10) -> dict:
    """The c2 prompt alone: the small LLMY model's 512-token prefill captured as
    one CUDA graph (PrefillGraph), replayed `reps` times inside the NVTX range
    "prefill_graph_timed" (for launch lists), CUDA events, median."""
    import numpy as np
    import torch

    from hybrid_llm_b200.config import small_llmy_config
    from hybrid_llm_b200.model import LoopedHybridModel, PrefillGraph
    from hybrid_llm_b200.weights import ModelWeights, synthetic_state_dict

    cfg = small_llmy_config()
    model = LoopedHybridModel(ModelWeights.from_state_dict(
        cfg, synthetic_state_dict(cfg, seed=0, device="cuda"), "cuda"))
    prompt = torch.from_numpy(np.random.default_rng(0).integers(0, cfg.vocab_size, (1, 512))).cuda()
    pg = PrefillGraph(model, 1, 512)
    for _ in range(3):
        pg.run(prompt)
    torch.cuda.synchronize()
    ts = []
    torch.cuda.nvtx.range_push("prefill_graph_timed")
    for _ in range(max(1, reps)):
        a, b = _events()
        a.record()
        pg.run(prompt)
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    torch.cuda.nvtx.range_pop()
    t = float(np.median(ts)) * 1e-3
    return {"workload": "small-llmy prefill, 512-token prompt, B=1, one CUDA graph replay",
            "ms": t * 1e3, "tok_s": 512 / t, "roofline": prefill_roofline(model, cfg, 512, t, p)}


def secondary_large_prefill(p: dict, reps: int = 2, chunk: int = 8, context: int = 4096,
                            global_batch: int = 64) -> dict:
    """Prompt forward of the large expert-parallel config on one GPU (d 2048,
    24 blocks, 64 experts top-8, 3 loops, vocab 64000): the 64 x 4096-token
    context as row chunks of `chunk` rows (prompt rows are independent, so a
    chunk of 8 does 1/8 of the work; at 8 rows every tensor stays below 2^31
    elements: 262,144 routed rows x 2048).  Eager forward (kernel-bound at
    32,768 tokens per call), last-position logits only, each call from a
    zeroed state; median over `reps` calls after one warm-up call."""
    import numpy as np
    import torch

    from hybrid_llm_b200 import kernels
    from hybrid_llm_b200.config import large_ep_config
    from hybrid_llm_b200.model import LoopedHybridModel
    from hybrid_llm_b200.state import RecurrentState
    from hybrid_llm_b200.weights import ModelWeights, synthetic_state_dict

    cfg = large_ep_config()
    model = LoopedHybridModel(ModelWeights.from_state_dict(
        cfg, synthetic_state_dict(cfg, seed=0, device="cuda"), "cuda"))
    g = torch.Generator(device="cpu").manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (chunk, context), generator=g).cuda()
    state = RecurrentState(cfg, chunk, "cuda")
    out = model.forward(ids, state=state, last_logits_only=True)
    torch.cuda.synchronize()
    kernels.check_device_status()
    ts = []
    torch.cuda.nvtx.range_push("large_prefill_timed")
    for _ in range(max(1, reps)):
        state.zero_()
        a, b = _events()
        a.record()
        out = model.forward(ids, state=state, last_logits_only=True)
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    torch.cuda.nvtx.range_pop()
    kernels.check_device_status()
    finite = bool(torch.isfinite(out.logits).all())
    t = float(np.median(ts)) * 1e-3
    tokens = chunk * context
    return {"workload": f"large-config prompt prefill, {context} tokens x {global_batch} rows as "
                        f"{global_batch // chunk} chunks of {chunk} rows, one GPU, eager forward",
            "chunk_rows": chunk, "ms_per_chunk": t * 1e3, "tok_s": tokens / t,
            "ms_for_global_batch": t * 1e3 * global_batch / chunk, "logits_finite": finite,
            "roofline": prefill_roofline(model, cfg, context, t, p, batch=chunk)}


def secondary_mhc(p: dict, reps: int = 10) -> dict:
    """Hyper-connection read / write around one sub-layer: 16384 tokens x D=1024
    with 4 fp32 streams (256 MB, above L2), L2 flushed before each timed call.
    Algorithmic bytes: write = streams read + written + bf16 update; read
    kernel = streams + bf16 and fp32 outputs (+ maps); theta GEMM = streams."""
    import numpy as np
    import torch

    from hybrid_llm_b200 import kernels
    from hybrid_llm_b200.weights import MhcBlock

    n, d, ns = 16384, 1024, 4
    nm = 2 * ns + ns * ns
    g = torch.Generator(device="cuda").manual_seed(0)
    rnd = lambda *shape, s=1.0: torch.randn(*shape, device="cuda", generator=g) * s
    blk = MhcBlock(theta=rnd(nm, ns * d, s=0.02).contiguous(), stream_scale=1 + rnd(ns, d, s=0.1),
                   ln_w=1 + rnd(d, s=0.1), ln_b=rnd(d, s=0.1),
                   bias=torch.cat([rnd(2 * ns, s=0.1), (torch.eye(ns, device="cuda") * 4).reshape(-1)]),
                   scalars=torch.tensor([0.3, 0.3, 0.3, 0.3], device="cuda"))
    norm_w = 1 + rnd(d, s=0.1)
    streams = rnd(n, ns * d)
    upd = rnd(n, d).bfloat16()
    maps = torch.empty(n, nm, device="cuda")
    ob = torch.empty(n, d, dtype=torch.bfloat16, device="cuda")
    of = torch.empty(n, d, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    iters = 10

    def read_kernel(raw):
        kernels._native.call("llmyb_mhc_read", streams.data_ptr(), n, ns, d, raw.data_ptr(),
                             raw.stride(0), raw.stride(1), blk.bias.data_ptr(), blk.scalars.data_ptr(), blk.ln_w.data_ptr(),
                             blk.ln_b.data_ptr(), norm_w.data_ptr(), 1e-6, iters, maps.data_ptr(),
                             ob.data_ptr(), of.data_ptr(), kernels._stream())

    raw = torch.mm(streams, blk.theta.t())
    parts = {"write": lambda: kernels.mhc_write(streams, ns, blk, maps, upd),
             "theta_gemm": lambda: torch.mm(streams, blk.theta.t(), out=raw),
             "read": lambda: read_kernel(raw)}
    sd4 = n * ns * d * 4
    alg = {"write": 2 * sd4 + n * d * 2, "theta_gemm": sd4 + n * nm * 4,
           "read": sd4 + n * nm * 8 + n * d * 6}
    for f in parts.values():
        for _ in range(3):
            f()
    res = {"workload": f"mHC read/write, {n} tokens x D={d}, {ns} fp32 streams, "
                       f"{iters} Sinkhorn iterations"}
    total = 0.0
    for name, f in parts.items():
        times = []
        for _ in range(max(1, reps)):
            flush.zero_()
            a, b = _events()
            a.record()
            f()
            b.record()
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b))
        t = float(np.median(times)) * 1e-3
        total += t
        gbs = alg[name] / t / 1e9
        res[f"{name}_us"] = t * 1e6
        res[f"{name}_gbs"] = gbs
        res[f"{name}_frac_of_hbm"] = gbs / p["hbm_gbs"]
    res["sublayer_us"] = total * 1e6
    res["algorithmic_bytes"] = alg
    return res


def secondary_prefill(p: dict, reps: int = 5, batch: int = 8) -> dict:
    """Long-context prefill kernels: banded attention and the GDN chunked scan
    (batch 8 is the workload; a smaller batch serves kernel profiles)."""
    import numpy as np
    import torch

    from hybrid_llm_b200 import kernels

    b, t, h, d, w = batch, 8192, 16, 128, 1024
    g = torch.Generator(device="cuda").manual_seed(1)
    q, k, v = (torch.randn(b, t, h, d, device="cuda", generator=g).bfloat16() for _ in range(3))
    out = torch.empty_like(q)
    for _ in range(3):
        kernels.banded_attention(q, k, v, w, out=out)
    times = []
    for _ in range(max(1, reps)):
        a, e_ = _events()
        a.record()
        kernels.banded_attention(q, k, v, w, out=out)
        e_.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(e_))
    ta = float(np.median(times)) * 1e-3
    pairs = w * (w + 1) / 2 + (t - w) * w
    attn_flops = 4.0 * d * pairs * b * h
    del out
    qn = torch.nn.functional.normalize(q.float(), dim=-1).bfloat16()
    kn = torch.nn.functional.normalize(k.float(), dim=-1).bfloat16()
    del q, k
    beta = torch.rand(b, t, h, device="cuda", generator=g).bfloat16()
    gate = torch.rand(b, t, h, d, device="cuda", generator=g).bfloat16()
    la = -0.1 * torch.rand(b, t, h, device="cuda", generator=g)
    st = torch.zeros(b, h, d, d, device="cuda")
    o = torch.empty_like(v)
    need = int(kernels._native.lib().llmyb_gdn_prefill_scratch_bytes(b, t, h, d, d))
    scratch = torch.empty(need, dtype=torch.uint8, device="cuda")
    for _ in range(2):
        st.zero_()
        kernels.gdn_prefill(qn, kn, v, gate, beta, st, log_alpha=la, out=o, scratch=scratch)
    times = []
    for _ in range(max(1, reps)):
        st.zero_()
        a, e_ = _events()
        a.record()
        kernels.gdn_prefill(qn, kn, v, gate, beta, st, log_alpha=la, out=o, scratch=scratch)
        e_.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(e_))
    tg = float(np.median(times)) * 1e-3
    gdn_bytes = b * t * h * (4 * d * 2 + 2 + 4) + 2 * b * h * d * d * 4
    return {"workload": f"B={b} T=8192 H=16 Dh=128: banded attention W=1024; GDN chunk-64 scan K=V=128",
            "banded_attention_ms": ta * 1e3, "banded_attention_tflops": attn_flops / ta / 1e12,
            "banded_attention_frac_of_bf16_peak": attn_flops / ta / 1e12 / p["bf16_tflops"],
            "gdn_scan_ms": tg * 1e3, "gdn_scan_gbs": gdn_bytes / tg / 1e9,
            "gdn_scan_frac_of_hbm": gdn_bytes / tg / 1e9 / p["hbm_gbs"],
            "prefill_tok_s": b * t / (ta + tg)}


def ep_decode_bytes_per_step(cfg, batch_local: int, world: int, weights) -> float:
    """Algorithmic HBM bytes one rank touches per decode step of the large
    expert-parallel config: its expert shard (every local expert is routed
    to at batch 64 x top-8 over 64 experts), the dense block weights (kept on
    every rank), the KV windows and GDN states of its own sequences, the head."""
    d = cfg.d_model
    nb = lambda t: t.numel() * t.element_size()
    dense = 0
    for blk in weights.blocks:
        m = blk.mixer
        dense += (nb(m.w_in) + nb(m.w_out) + nb(m.conv)) if blk.kind == "gdn" else \
            (nb(m.w_in) + nb(m.w_o))
        dense += nb(blk.moe.router) + nb(blk.moe.w13) + nb(blk.moe.w2)
    dense *= cfg.num_loops
    n_csa = sum(1 for j in range(cfg.n_blocks) if cfg.block_kind(j) == "csa") * cfg.num_loops
    n_gdn = cfg.n_blocks * cfg.num_loops - n_csa
    kv = batch_local * n_csa * cfg.csa_window * (cfg.csa_heads * cfg.csa_head_dim + d) * 2
    gdn_state = batch_local * n_gdn * cfg.gdn_heads * cfg.gdn_key_dim * cfg.gdn_value_dim * 4 * 2
    head = cfg.vocab_size * d * 2 + d * d * 2
    return float(dense + kv + gdn_state + head)


def secondary_ep_decode(p: dict, steps: int = 10, warmup: int = 3, global_batch: int = 64,
                        context: int = 4096, exchange: str = "p2p") -> dict:
    """Large expert-parallel config decode: d 2048, 24 blocks, 64 experts top-8,
    3 loops, vocab 64000, global batch 64 split over the ranks; experts sharded
    64/W per rank (ExpertParallel, all-to-all over NCCL) for W > 1.  The
    4096-token context is a synthetic recurrent state (RecurrentState.
    fill_synthetic): decode cost does not depend on the context's values.
    exchange "p2p" (peer-memory, the step replayed as one CUDA graph) or
    "nccl" (all_to_all_single, eager).  Collective when torch.distributed is
    initialised: every rank calls it."""
    import torch
    import torch.distributed as dist

    from hybrid_llm_b200 import kernels
    from hybrid_llm_b200.config import large_ep_config
    from hybrid_llm_b200.expert_parallel import ExpertParallel
    from hybrid_llm_b200.model import GreedyDecoder, LoopedHybridModel, PrefillGraph
    from hybrid_llm_b200.state import RecurrentState
    from hybrid_llm_b200.weights import ModelWeights, synthetic_state_dict

    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    cfg = large_ep_config()
    bl = global_batch // world
    ep = None
    if world > 1:
        ep = ExpertParallel(cfg.moe_experts, cfg.moe_top_k, cfg.d_model, cfg.moe_hidden, bl,
                            exchange=exchange)
    use_graph = ep is None or exchange == "p2p"
    weights = ModelWeights.from_state_dict(cfg, synthetic_state_dict(cfg, seed=0, device="cuda"),
                                           "cuda", expert_range=None if ep is None else ep.expert_range)
    model = LoopedHybridModel(weights, ep=ep)
    state = RecurrentState(cfg, bl, "cuda")
    state.fill_synthetic(context, seed=rank)
    dec = GreedyDecoder(model, state, use_graph=use_graph)
    g = torch.Generator(device="cpu").manual_seed(rank)
    dec.prime(torch.randint(0, cfg.vocab_size, (bl,), generator=g).cuda())
    # graph replays launch nothing through the library: count one eager step
    n0 = kernels.launch_count()
    dec.use_graph = False
    dec.step()
    per_step = kernels.launch_count() - n0
    dec.use_graph = use_graph
    for _ in range(warmup):  # the first graph step captures
        dec.step()
    torch.cuda.synchronize()
    n0 = kernels.launch_count()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = _events()
    torch.cuda.nvtx.range_push("ep_decode_timed")
    a.record()
    for _ in range(steps):
        dec.step()
    b.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_ms = a.elapsed_time(b)
    launches = per_step if use_graph else (kernels.launch_count() - n0) // steps
    kernels.check_device_status()
    if world > 1:
        tt = torch.tensor([t_ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_ms = float(tt.item())
    del dec
    if ep is not None:
        dist.barrier()
        ep.close()
    step_s = t_ms * 1e-3 / steps
    touched = ep_decode_bytes_per_step(cfg, bl, world, weights)
    achieved = touched / step_s / 1e9
    return {"workload": "large expert-parallel config: d 2048, 24 blocks, 64 experts top-8, "
                        "3 loops, vocab 64000, batch 64, 4096-token synthetic context",
            "n_gpus": world, "batch_per_rank": bl, "parallelism": f"ep{world}" if world > 1 else
            "single", "exchange": None if world == 1 else (
                "peer-memory stores over NVLink (CUDA IPC), flags" if exchange == "p2p"
                else "NCCL all_to_all_single"),
            "graph": use_graph, "tok_s": global_batch / step_s, "ms_per_step": step_s * 1e3,
            "scaling": "strong (global batch 64 split over the ranks)",
            "llmyb_launches_per_step": launches,
            "hbm_bytes_per_step_per_rank": touched, "achieved_gbs_per_rank": achieved,
            "frac_of_hbm": achieved / p["hbm_gbs"]}


def run_ours(args) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist

    from hybrid_llm_b200 import kernels
    from hybrid_llm_b200.config import small_llmy_config
    from hybrid_llm_b200.model import GreedyDecoder, LoopedHybridModel, PrefillGraph
    from hybrid_llm_b200.weights import ModelWeights, synthetic_state_dict

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    p = peaks()
    cfg = small_llmy_config()
    bsz, prompt_len = 1, 512
    model = LoopedHybridModel(ModelWeights.from_state_dict(
        cfg, synthetic_state_dict(cfg, seed=0, device="cuda"), "cuda"))
    prompt = torch.from_numpy(np.random.default_rng(0).integers(0, cfg.vocab_size, (bsz, prompt_len))).cuda()

    # prefill (timed separately: prompt tokens/s), eager and as one graph replay
    model.forward(prompt, last_logits_only=True)
    torch.cuda.synchronize()
    a, b = _events()
    a.record()
    out = model.forward(prompt, last_logits_only=True)
    b.record()
    torch.cuda.synchronize()
    prefill_eager_s = a.elapsed_time(b) * 1e-3
    pgraph = PrefillGraph(model, bsz, prompt_len)
    ptimes = []
    for _ in range(5):
        a, b = _events()
        a.record()
        out = pgraph.run(prompt)
        b.record()
        torch.cuda.synchronize()
        ptimes.append(a.elapsed_time(b))
    prefill_s = float(np.median(ptimes)) * 1e-3

    dec = GreedyDecoder(model, out.state, use_graph=True)
    dec.prime(out.logits[:, -1].float().argmax(-1))
    n0 = kernels.launch_count()
    dec.capture()
    launches_capture = kernels.launch_count() - n0
    # capture() runs one eager warm-up step then captures one step
    launches_per_step = launches_capture // 2
    for _ in range(args.warmup):
        dec.step()
    torch.cuda.synchronize()

    clocks = ClockSampler(local)
    with clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        a, b = _events()
        torch.cuda.nvtx.range_push("decode_timed")
        a.record()
        for _ in range(args.steps):
            dec.step()
        b.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    t_ms = a.elapsed_time(b)
    if world > 1:
        tt = torch.tensor([t_ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_ms = float(tt.item())
    value = bsz * args.steps * world / (t_ms * 1e-3)

    # e2e: public decode API with a pinned-host token round trip per step: the
    # token in, the step and the token + log-probability out are one graph
    # replay (GreedyDecoder.step_host), then the host waits and feeds the token back
    dec.step_host()  # captures the host-I/O graph (one untimed step)
    host_in, host_out, host_lp = dec.host_in, dec.host_out, dec.host_lp
    torch.cuda.synchronize()
    host_in.copy_(host_out)
    a, b = _events()
    a.record()
    for _ in range(args.steps):
        dec.step_host()
        torch.cuda.current_stream().synchronize()
        host_in.copy_(host_out)
    b.record()
    torch.cuda.synchronize()
    e2e_ms = a.elapsed_time(b)
    if world > 1:
        tt = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt.item())
    e2e = {"value": bsz * args.steps * world / (e2e_ms * 1e-3), "unit": "tok/s",
           "h2d_bytes_per_step": host_in.numel() * 8,
           "d2h_bytes_per_step": host_out.numel() * 8 + host_lp.numel() * 4}

    # roofline of the whole step (weights and state touched per token) and of
    # the dominant kernel of the step's launch list
    touched = decode_bytes_per_step(model, cfg)
    achieved = touched / (t_ms * 1e-3 / args.steps) / 1e9
    step_roofline = {"bound": "hbm", "achieved": achieved, "peak": p["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / p["hbm_gbs"],
                     "what": "whole decode step (one CUDA graph); algorithmic bytes = weights "
                             "and state touched per token",
                     "algorithmic_bytes_per_step": touched}
    from hybrid_llm_b200 import persistent
    if model.decode_persistent and persistent.supported(model, bsz):
        roofline = persistent_roofline(model, dec.state, p)
        touched = decode_bytes_per_step(model, cfg, folded=True)
        achieved = touched / (t_ms * 1e-3 / args.steps) / 1e9
        step_roofline.update(achieved=achieved, frac=achieved / p["hbm_gbs"],
                             algorithmic_bytes_per_step=touched)
    else:
        roofline = out_router_roofline(model, p)

    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform token ids, N(0,0.02) random-init weights)",
        "config": {"workload": WORKLOAD, "batch": bsz, "prompt_len": prompt_len,
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": "no flush: >1 GB of weights, about 0.3 GB touched per step (> 126 MB L2)"},
        "e2e": e2e, "gpu_launches": launches_per_step * args.steps, "roofline": roofline,
        "step_roofline": step_roofline,
        "clocks": clocks.summary(), "prefill_tok_s_c2": bsz * prompt_len / prefill_s,
        "prefill_c2_note": "one CUDA graph replay of the 512-token forward (median of 5); "
                           "eager forward (host launch cost included) in prefill_eager_ms",
        "prefill_eager_ms": prefill_eager_s * 1e3,
        "prefill_roofline": prefill_roofline(model, cfg, prompt_len, prefill_s, p),
    }
    del dec, out, model, pgraph
    torch.cuda.empty_cache()
    secondary = {}
    if not args.no_ep:  # every rank: expert parallel over the whole group when N > 1
        secondary["large_ep_decode"] = secondary_ep_decode(p, steps=10, warmup=3)
        torch.cuda.empty_cache()
    if rank == 0 and world == 1 and not args.no_secondary:
        secondary["single_block"] = secondary_block(p)
        secondary["moe_layer"] = secondary_moe(p)
        secondary["long_prefill"] = secondary_prefill(p)
        secondary["large_prefill"] = secondary_large_prefill(p)
        torch.cuda.empty_cache()
        secondary["mhc"] = secondary_mhc(p)
        secondary["sampling_router"] = secondary_sampling_router(p)
    if secondary:
        line["secondary"] = secondary
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_decode_baseline(steps=3, warmup=1)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def prefill_roofline(model, cfg, tokens: int, seconds: float, p: dict, batch: int = 1) -> dict:
    """Roofline of a prefill of `batch` rows of `tokens` ids: the algorithmic HBM bytes
    (every dense weight and every expert once per loop -- at 512 tokens and
    top-2 each of the 16 experts receives rows --, the LM head row block of
    the last token) against the algorithmic FLOPs (2 x the weights each token
    uses, the CSA scores and PV over each token's window, the GDN state
    update and readout); the bound is whichever takes longer at the measured
    peaks."""
    d, nl = cfg.d_model, cfg.num_loops
    nb = lambda t: t.numel() * t.element_size()
    dense_bytes = dense_params = 0
    expert_bytes = 0
    attn_flops = 0.0
    keys = sum(min(t + 1, cfg.csa_window) for t in range(tokens))
    for blk in model.w.blocks:
        m = blk.mixer
        if blk.kind == "gdn":
            mats = (m.w_in, m.w_out)
            attn_flops += tokens * 4.0 * cfg.gdn_heads * cfg.gdn_key_dim * cfg.gdn_value_dim * 2
        else:
            mats = (m.w_in, m.local_out, m.out)
            hd = cfg.csa_heads * cfg.csa_head_dim
            attn_flops += 2.0 * keys * (hd + d)
        for w in mats + (blk.moe.router,):
            dense_bytes += nb(w)
            dense_params += w.numel()
        expert_bytes += nb(blk.moe.w13) + nb(blk.moe.w2)
    act_expert = 3 * cfg.moe_hidden * d * cfg.moe_top_k * cfg.n_blocks
    flops = batch * (nl * (2.0 * tokens * (dense_params + act_expert) + attn_flops) +
                     2.0 * cfg.vocab_size * d)
    bytes_ = nl * (dense_bytes + expert_bytes) + cfg.vocab_size * d * 2 + batch * tokens * d * 2
    t_hbm = bytes_ / (p["hbm_gbs"] * 1e9)
    t_tc = flops / (p["bf16_tflops"] * 1e12)
    t_roof = max(t_hbm, t_tc)
    return {"bound": "hbm" if t_hbm >= t_tc else "tensor", "tokens": tokens, "batch": batch,
            "algorithmic_bytes": bytes_, "algorithmic_flops": flops,
            "t_roofline_ms": t_roof * 1e3, "t_ms": seconds * 1e3, "frac": t_roof / seconds,
            "frac_of_sustained_peaks": max(
                t_hbm, flops / (p.get("bf16_tflops_sustained", p["bf16_tflops"]) * 1e12)) / seconds,
            "achieved_gbs": bytes_ / seconds / 1e9, "achieved_tflops": flops / seconds / 1e12}


def decode_bytes_per_step(model, cfg, folded: bool = False) -> float:
    """Algorithmic HBM bytes of one decode token at B=1: every dense weight once,
    the routed experts (top-k of E per block and loop), the KV window and GDN
    state of every block-loop, the tied LM head.  folded: the persistent step's
    CSA input projection carries the output projection in its value rows, so
    no separate output matrix is read."""
    d = cfg.d_model
    dense = 0
    nb = lambda t: t.numel() * t.element_size()
    for blk in model.w.blocks:
        m = blk.mixer
        if blk.kind == "gdn":
            dense += nb(m.w_in) + nb(m.w_out) + nb(m.conv)
        else:
            # decode uses the pre-multiplied output matrix, or (folded) none at all
            dense += nb(m.w_in) + (0 if folded else nb(m.w_o))
        dense += nb(blk.moe.router)
    dense *= cfg.num_loops
    expert = 3 * cfg.moe_hidden * d * 2 * cfg.moe_top_k * cfg.n_blocks * cfg.num_loops
    n_csa = sum(1 for j in range(cfg.n_blocks) if cfg.block_kind(j) == "csa") * cfg.num_loops
    n_gdn = cfg.n_blocks * cfg.num_loops - n_csa
    kv = n_csa * cfg.csa_window * (cfg.csa_heads * cfg.csa_head_dim + d) * 2
    gdn_state = n_gdn * cfg.gdn_heads * cfg.gdn_key_dim * cfg.gdn_value_dim * 4 * 2
    head = cfg.vocab_size * d * 2 + d * d * 2
    return float(dense + expert + kv + gdn_state + head)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ep", action="store_true",
                    help="skip the large expert-parallel decode measurement")
    ap.add_argument("--ep-exchange", choices=["p2p", "nccl"], default="p2p",
                    help="expert-parallel exchange of --only ep_decode")
    ap.add_argument("--only", choices=["single_block", "moe_layer", "long_prefill", "ep_decode",
                                       "mhc", "sampling_router", "prefill_c2", "large_prefill"],
                    default=None,
                    help="run one secondary workload alone (used for kernel profiles)")
    ap.add_argument("--prefill-batch", type=int, default=8,
                    help="batch of the long-context prefill workload (profiles use 1)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.only == "ep_decode":
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        if int(os.environ.get("WORLD_SIZE", "1")) > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        res = secondary_ep_decode(peaks(), steps=args.steps, warmup=args.warmup,
                                  exchange=args.ep_exchange)
        if not dist.is_initialized() or dist.get_rank() == 0:
            print(json.dumps({"only": args.only, **res}), flush=True)
        if dist.is_initialized():
            dist.destroy_process_group()
    elif args.only:
        import torch
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        if args.only == "long_prefill":
            res = secondary_prefill(peaks(), reps=args.steps, batch=args.prefill_batch)
        elif args.only == "single_block":
            res = secondary_block(peaks(), reps=args.steps)
        elif args.only == "prefill_c2":
            res = secondary_prefill_c2(peaks())
        elif args.only == "large_prefill":
            res = secondary_large_prefill(peaks(), reps=args.steps, chunk=args.prefill_batch)
        elif args.only == "sampling_router":
            res = secondary_sampling_router(peaks())
        elif args.only == "mhc":
            res = secondary_mhc(peaks(), reps=args.steps)
        else:
            res = secondary_moe(peaks(), reps=args.steps)
        print(json.dumps({"only": args.only, **res}), flush=True)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
