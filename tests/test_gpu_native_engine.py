"""GPU: the native engine (include/llmy.h, csrc/engine.cu) on `.llmy` files.

* The converter's fixture (tests/golden/tiny_model.llmy, window 16 so the
  rings wrap) stepped token by token through llmy_decode against the fp64
  oracle on the file's own weights, routing-aware (tests/route_parity.py:
  the oracle forced onto the experts the engine reports through
  llmyb_engine_routes; every differing choice a near tie): every prompt
  position and six teacher-forced decode steps.
* The same and a 512-wide two-block model written with llmy_format against
  the Python model's persistent decode step (the same kernel behind torch
  tensors): logits within 2e-2 of max |ref|, the same experts except at most
  one near tie per step.
* The API: getters, llmy_prefill equal to the steps it stands for, host and
  device logits buffers, fewer loops, set_num_loops, reset, an out-of-range
  token reported, and a C program that generates through the engine with no
  Python in the process.
"""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

import native_llmy as nl

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
FIXTURE = ROOT / "tests" / "golden" / "tiny_model.llmy"
LOGIT_REL = 3e-2
STEP_REL = 2e-2


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


class Engine:
    """One loaded model and one state, with host logits."""

    def __init__(self, path, loops: int | None = None):
        self.L = nl.lib()
        self.m = self.L.llmy_load(str(path).encode())
        assert self.m, f"llmy_load failed for {path}"
        if loops is not None:
            self.L.llmy_set_num_loops(self.m, loops)
        self.s = self.L.llmy_state_new(self.m)
        assert self.s
        self.v = self.L.llmy_vocab_size(self.m)
        self.logits = np.zeros(self.v, dtype=np.float32)
        nb_k = 64 * 8 * 8
        self.idx = np.zeros(nb_k, dtype=np.int32)

    def decode(self, tok: int, pos: int, loops: int = 0) -> np.ndarray:
        self.L.llmy_decode(self.m, self.s, int(tok), int(pos), loops, nl.fptr(self.logits))
        return self.logits.copy()

    def routes(self, n_blocks: int, k: int) -> np.ndarray:
        n = self.L.llmyb_engine_routes(self.s, self.idx.ctypes.data, None, self.idx.size)
        assert n > 0 and n % (n_blocks * k) == 0, n
        return self.idx[:n].reshape(-1, n_blocks, k).copy()

    def close(self):
        self.L.llmy_state_free(self.s)
        self.L.llmy_free(self.m)


def _file_model(path):
    """The oracle's configuration and per-expert weights of a `.llmy` file."""
    import re
    from hybrid_llm_b200 import llmy_format
    from hybrid_llm_b200.config import HybridConfig
    f = llmy_format.read_llmy(path)
    cfg = HybridConfig.from_v6(f.config)
    sd = {}
    for name, t in f.tensors.items():
        mt = re.match(r"^(.+\.experts)\.([a-z_]+\.weight)$", name)
        if mt:
            for e in range(t.shape[0]):
                sd[f"{mt.group(1)}.{e}.{mt.group(2)}"] = t[e].clone()
        else:
            sd[name] = t.clone()
    f.close()
    return cfg, sd


def test_native_engine_vs_oracle_routing_aware(cuda):
    import route_parity
    from oracle.model import OracleModel
    cfg, sd = _file_model(FIXTURE)
    orc = OracleModel(cfg, sd)
    eng = Engine(FIXTURE)
    nb, k = cfg.n_blocks, cfg.moe_top_k
    rng = np.random.default_rng(21)
    prompt = rng.integers(0, cfg.vocab_size, size=40)
    got, step_routes = [], []
    for t, tok in enumerate(prompt):
        got.append(eng.decode(tok, t))
        step_routes.append(eng.routes(nb, k))
    # the oracle's forward over the prompt makes one MoE call per (loop, block)
    forced = [np.stack([r[i, j] for r in step_routes]) for i in range(cfg.num_loops)
              for j in range(nb)]
    (ref, st), log = route_parity._forced(orc, forced, orc.forward, prompt[None])
    mism, worst = route_parity.route_mismatches(log, forced, 2e-2)
    errs = [_rel(got[t], ref[0, t]) for t in range(prompt.size)]
    print("prompt: mismatches", mism, "worst tie", worst, "worst rel", max(errs))
    assert max(errs) < LOGIT_REL, (int(np.argmax(errs)), max(errs))
    toks = rng.integers(0, cfg.vocab_size, size=6)
    for s, tok in enumerate(toks):
        out = eng.decode(tok, prompt.size + s)
        r = eng.routes(nb, k)
        forced = [r[i, j][None] for i in range(cfg.num_loops) for j in range(nb)]
        (ref_s, st), log = route_parity._forced(orc, forced, orc.decode_step, np.array([tok]), st)
        route_parity.route_mismatches(log, forced, 2e-2)
        assert _rel(out, ref_s[0]) < LOGIT_REL, (s, _rel(out, ref_s[0]))
    eng.close()


def _compare_with_python(path, steps: int, seed: int):
    from hybrid_llm_b200 import kernels, persistent
    from hybrid_llm_b200.model import LoopedHybridModel
    from hybrid_llm_b200.state import RecurrentState
    from hybrid_llm_b200.weights import ModelWeights
    pm = LoopedHybridModel(ModelWeights.from_llmy(path, "cuda"))
    assert persistent.supported(pm, 1)
    cfg = pm.cfg
    st = RecurrentState(cfg, 1, "cuda")
    eng = Engine(path)
    rng = np.random.default_rng(seed)
    toks = rng.integers(0, cfg.vocab_size, size=steps)
    worst, flips_total = 0.0, 0
    for t, tok in enumerate(toks):
        a = eng.decode(tok, t)
        ra = eng.routes(cfg.n_blocks, cfg.moe_top_k)
        pm.route_log = []
        b = pm.decode_step(torch.tensor([int(tok)], device="cuda"), st)[0].float().cpu().numpy()
        rb = torch.cat(pm.route_log).cpu().numpy().reshape(ra.shape)
        pm.route_log = None
        e = _rel(a, b)
        worst = max(worst, e)
        assert e < STEP_REL, (t, e)
        flips = int((np.sort(ra, -1) != np.sort(rb, -1)).any(-1).sum())
        assert flips <= 1, (t, flips)
        flips_total += flips
    kernels.check_device_status()
    eng.close()
    return worst, flips_total


def test_native_engine_matches_python_persistent_tiny(cuda):
    print("tiny", _compare_with_python(FIXTURE, 40, 3))


def test_native_engine_matches_python_persistent_single_block(cuda, tmp_path):
    """A 512-wide csa_moe + gdn_moe model (vocab 32000, 8 experts of 1024, the
    bench's single-block shape) written by llmy_format from synthetic weights."""
    import inputs
    from hybrid_llm_b200 import llmy_format
    from hybrid_llm_b200.config import single_block_config
    from hybrid_llm_b200.weights import synthetic_state_dict
    cfg = single_block_config()
    sd = {k: (v.bfloat16() if v.dim() >= 2 else v.float())
          for k, v in synthetic_state_dict(cfg, seed=0).items()}
    path = tmp_path / "single.llmy"
    llmy_format.write_llmy(path, inputs.v6_mapping(cfg), sd)
    print("single block", _compare_with_python(path, 24, 4))


def test_native_engine_api(cuda, capfd):
    import dataclasses
    from hybrid_llm_b200.model import LoopedHybridModel
    from hybrid_llm_b200.state import RecurrentState
    from hybrid_llm_b200.weights import ModelWeights
    eng = Engine(FIXTURE)
    L, m, s, v = eng.L, eng.m, eng.s, eng.v
    assert (v, L.llmy_d_model(m), L.llmy_num_loops(m), L.llmy_max_loops(m),
            L.llmy_mhc_streams(m)) == (256, 128, 2, 2, 1)
    prompt = (np.arange(30, dtype=np.int32) * 37) % v
    # prefill = the same steps with the head skipped before the last
    pre = np.zeros(v, dtype=np.float32)
    L.llmy_prefill(m, s, nl.iptr(prompt), prompt.size, nl.fptr(pre))
    assert L.llmy_last_executed_loops(s) == 2
    e2 = Engine(FIXTURE)
    for t, tok in enumerate(prompt):
        by_steps = e2.decode(tok, t)
    assert np.array_equal(pre, by_steps)
    # device logits buffer
    dev = torch.zeros(v, dtype=torch.float32, device="cuda")
    L.llmy_decode(m, s, 5, prompt.size, 0, nl.fptr(dev))
    host = e2.decode(5, prompt.size)
    assert np.array_equal(dev.cpu().numpy(), host)
    # reset replays the prompt to the same logits
    L.llmy_state_reset(s)
    again = np.zeros(v, dtype=np.float32)
    L.llmy_prefill(m, s, nl.iptr(prompt), prompt.size, nl.fptr(again))
    assert np.array_equal(again, pre)
    # one loop per step on a two-loop state = a one-loop model's persistent step
    L.llmy_state_reset(s)
    w = ModelWeights.from_llmy(FIXTURE, "cuda")
    w.cfg = dataclasses.replace(w.cfg, num_loops=1)
    pm = LoopedHybridModel(w)
    st = RecurrentState(pm.cfg, 1, "cuda")
    for t, tok in enumerate(prompt[:20]):
        a = eng.decode(tok, t, loops=1)
        assert L.llmy_last_executed_loops(s) == 1
        b = pm.decode_step(torch.tensor([int(tok)], device="cuda"), st)[0].float().cpu().numpy()
        assert _rel(a, b) < STEP_REL, (t, _rel(a, b))
    # an out-of-range token is clamped by the kernel and reported
    capfd.readouterr()
    eng.decode(v + 5, 20)
    err = capfd.readouterr().err
    assert "[llmy_decode] device status 1" in err, err
    assert np.isfinite(eng.decode(3, 21)).all()
    assert "[llmy_decode]" not in capfd.readouterr().err
    # loops above the state's slots are capped
    L.llmy_set_num_loops(m, 3)
    eng.decode(3, 22)
    assert L.llmy_last_executed_loops(s) == 2
    assert "the state holds 2 loops" in capfd.readouterr().err
    e2.close()
    eng.close()


C_PROGRAM = r"""
#include <stdio.h>
#include <stdlib.h>
#include "llmy.h"
int main(int argc, char** argv) {
  llmy_model* m = llmy_load(argv[1]);
  if (!m) return 2;
  llmy_state* s = llmy_state_new(m);
  if (!s) return 3;
  const int v = llmy_vocab_size(m), n = 12;
  int32_t prompt[12];
  for (int i = 0; i < n; ++i) prompt[i] = (i * 7) % v;
  float* logits = (float*)malloc(sizeof(float) * v);
  llmy_prefill(m, s, prompt, n, logits);
  uint64_t rng = 1;
  for (int step = 0; step < 10; ++step) {
    const int32_t tok = llmy_sample(logits, v, 0.8f, 40, 0.95f, 1.1f, prompt, n, &rng);
    printf("%d\n", tok);
    llmy_decode(m, s, tok, n + step, 0, logits);
  }
  free(logits);
  llmy_state_free(s);
  llmy_free(m);
  return 0;
}
"""


def test_c_program_generates_without_python(cuda, tmp_path):
    """A C caller of the reference API (prefill, sample, decode loop), built
    with gcc against include/llmy.h and libllmyb.so: the same tokens as the
    same loop driven through ctypes."""
    from hybrid_llm_b200 import _native
    src = tmp_path / "gen.c"
    src.write_text(C_PROGRAM)
    exe = tmp_path / "gen"
    lib_dir = Path(_native.LIB_PATH).parent
    subprocess.run(["gcc", "-O2", "-I", str(ROOT / "include"), str(src), "-o", str(exe),
                    "-L", str(lib_dir), "-lllmyb", f"-Wl,-rpath,{lib_dir}"], check=True)
    res = subprocess.run([str(exe), str(FIXTURE)], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stderr
    got = [int(x) for x in res.stdout.split()]
    eng = Engine(FIXTURE)
    L, v = eng.L, eng.v
    prompt = (np.arange(12, dtype=np.int32) * 7) % v
    L.llmy_prefill(eng.m, eng.s, nl.iptr(prompt), 12, nl.fptr(eng.logits))
    rng = C.c_uint64(1)
    want = []
    for step in range(10):
        tok = L.llmy_sample(nl.fptr(eng.logits), v, 0.8, 40, 0.95, 1.1, nl.iptr(prompt), 12,
                            C.byref(rng))
        want.append(tok)
        eng.decode(tok, 12 + step)
    eng.close()
    assert got == want, (got, want)
