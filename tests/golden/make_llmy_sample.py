"""Golden vectors for the engine's host sampler, made by the reference's own code.

Run in a container that has the reference checkout::

    python tests/golden/make_llmy_sample.py

Builds the reference ``llmy_sample`` (llmy_cuda/src/llmy.cpp:132-202) with
oracle/build_ref.py, calls it on seeded random logits over a grid of
temperature / top-k / top-p / repetition-penalty settings (vocabulary sizes 1
to 32000, out-of-range and repeated recent ids included) and writes
``tests/golden/llmy_sample.npz``: the concatenated logits and recent ids with
per-case offsets, the settings, the rng state before and after, and the token.
Cases whose top-k boundary has equal logits are excluded: the reference leaves
their order open.  Nothing at test time reads the reference.
"""
from __future__ import annotations

import ctypes
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle import build_ref  # noqa: E402


def main() -> None:
    path = build_ref.build_ref()
    if path is None:
        raise SystemExit("reference checkout not found")
    lib = ctypes.CDLL(str(path), mode=os.RTLD_LAZY)
    fn = lib.llmy_sample
    fn.restype = ctypes.c_int32
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_float, ctypes.c_int32, ctypes.c_float,
                   ctypes.c_float, ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(ctypes.c_uint64)]
    rng = np.random.default_rng(2024)
    logits, recents = [], []
    rec = {k: [] for k in ("vocab", "logit_off", "temperature", "top_k", "top_p", "rep",
                           "recent_off", "n_recent", "state_in", "state_out", "token")}
    lo = ro = 0
    while len(rec["token"]) < 96:
        vocab = int(rng.choice([1, 2, 7, 100, 300, 1000, 2000])) if len(rec["token"]) < 95 else 32000
        lg = (rng.normal(size=vocab) * rng.choice([0.5, 3.0, 10.0])).astype(np.float32)
        if np.unique(lg).size != vocab:
            continue
        temp = float(rng.choice([0.0, -1.0, 0.3, 0.8, 1.0, 1.7]))
        top_k = int(rng.choice([0, 1, 5, 50, 256, 300, 100000]))
        top_p = float(rng.choice([0.0, 0.5, 0.9, 0.95, 1.0]))
        rep = float(rng.choice([1.0, 1.1, 1.3, 0.9]))
        recent = rng.integers(-3, vocab + 3, size=int(rng.integers(0, 24))).astype(np.int32)
        if recent.size:
            recent[-1] = recent[0]  # a repeated id is penalised again
        s0 = int(rng.integers(1, 2**63, dtype=np.int64))
        st = ctypes.c_uint64(s0)
        tok = fn(lg.ctypes.data, vocab, temp, top_k, top_p, rep,
                 recent.ctypes.data if recent.size else None, recent.size, ctypes.byref(st))
        for k, v in (("vocab", vocab), ("logit_off", lo), ("temperature", temp), ("top_k", top_k),
                     ("top_p", top_p), ("rep", rep), ("recent_off", ro),
                     ("n_recent", recent.size), ("state_in", s0), ("state_out", st.value),
                     ("token", tok)):
            rec[k].append(v)
        logits.append(lg)
        recents.append(recent)
        lo += vocab
        ro += recent.size
    out = {k: np.array(v, dtype=np.uint64 if k.startswith("state") else None)
           for k, v in rec.items()}
    out["logits"] = np.concatenate(logits)
    out["recent"] = np.concatenate(recents)
    np.savez_compressed(HERE / "llmy_sample.npz", **out)
    print(f"wrote {len(rec['token'])} cases to {HERE / 'llmy_sample.npz'}")


if __name__ == "__main__":
    main()
