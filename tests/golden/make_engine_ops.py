"""Golden vectors for the engine's device entry points, from the reference's own code.

Run in a container that has the reference checkout (``LLMY_REFERENCE``;
by default the directory ``reference`` beside this repository)::

    python tests/golden/make_engine_ops.py

Sinkhorn: model/layers/mhc.py:12-17 (``_sinkhorn_impl``) on seeded fp32 [N, 4, 4]
logits for 0, 1, 5 and 20 iterations.  One-token MoE: model/layers/moe.py:29-82
(``_moe_dispatch_fused``, the reference MoE on one token) in fp32 with seeded
weights; the gate/up weights are also stored in the engine's [E, 2H, D] layout
(gate rows, then up rows).  Writes ``tests/golden/engine_ops.npz``.  Nothing at
test time reads the reference.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("LLMY_REFERENCE",
                        Path(__file__).resolve().parents[2].parent / "reference"))

import torch  # noqa: E402


def main() -> None:
    if not REF.exists():
        raise SystemExit(f"reference checkout not found at {REF}")
    sys.path.insert(0, str(REF))
    from model.layers.mhc import _sinkhorn_impl
    from model.layers.moe import _moe_dispatch_fused

    rng = np.random.default_rng(11)
    out = {}
    logits = (rng.normal(size=(257, 4, 4)) * 2.0).astype(np.float32)
    out["sk_in"] = logits
    for it in (0, 1, 5, 20):
        out[f"sk_out_{it}"] = _sinkhorn_impl(torch.from_numpy(logits), it).numpy()

    e, d, h, k = 4, 32, 48, 3
    x = rng.normal(size=(1, d)).astype(np.float32)
    wg = (rng.normal(size=(e, h, d)) * 0.1).astype(np.float32)
    wu = (rng.normal(size=(e, h, d)) * 0.1).astype(np.float32)
    wd = (rng.normal(size=(e, d, h)) * 0.1).astype(np.float32)
    idx = np.array([[3, 0, 3]], dtype=np.int64)  # an expert picked twice
    prob = np.array([[0.5, 0.3, 0.2]], dtype=np.float32)
    y = _moe_dispatch_fused(torch.from_numpy(x), torch.from_numpy(idx), torch.from_numpy(prob),
                            torch.from_numpy(wg), torch.from_numpy(wu), torch.from_numpy(wd))
    out.update(moe_x=x[0], moe_idx=idx[0], moe_prob=prob[0],
               moe_gate_up=np.concatenate([wg, wu], axis=1), moe_down=wd,
               moe_out=y.numpy()[0])
    np.savez_compressed(HERE / "engine_ops.npz", **out)
    print(f"wrote {HERE / 'engine_ops.npz'}")


if __name__ == "__main__":
    main()
