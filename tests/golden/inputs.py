"""Seeded inputs shared by the golden generator and the tests.

The fixtures store only the reference's outputs (plus a checksum of the
inputs); both sides rebuild the inputs from these functions, so the committed
files stay small.
"""
from __future__ import annotations

import hashlib

import numpy as np


def checksum(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()[:16]


ROUTER_CASES = {"a": (512, 64, 32, 4), "b": (96, 64, 16, 2), "c": (64, 64, 64, 8)}


def router_case(tag: str):
    """hidden [1,N,D] fp32 and router logits weight [E,D] fp32."""
    n, d, e, k = ROUTER_CASES[tag]
    rng = np.random.default_rng(1000 + ord(tag))
    weight = rng.normal(0, 0.2, (e, d)).astype(np.float32)
    hidden = rng.normal(0, 1, (1, n, d)).astype(np.float32)
    return dict(hidden=hidden, weight=weight, k=k)


MOE_CASES = {"a": (96, 64, 8, 2, 32), "b": (40, 64, 8, 4, 32)}


def moe_case(tag: str):
    """flat [N,D], router logits [N,E], expert stacks (moe.py:119-125 layout)."""
    n, d, e, k, f = MOE_CASES[tag]
    rng = np.random.default_rng(2000 + ord(tag))
    return dict(
        flat=rng.normal(0, 1, (n, d)).astype(np.float32),
        logits=rng.normal(0, 1, (n, e)).astype(np.float32),
        w_gate=rng.normal(0, 0.05, (e, f, d)).astype(np.float32),
        w_up=rng.normal(0, 0.05, (e, f, d)).astype(np.float32),
        w_down=rng.normal(0, 0.05, (e, d, f)).astype(np.float32),
        k=k,
    )
