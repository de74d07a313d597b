"""Generate the ``.llmy`` fixture with the reference's own checkpoint converter.

Run in a container that has the reference checkout (``LLMY_REFERENCE``;
by default the directory ``reference`` beside this repository)::

    python tests/golden/make_llmy.py

Builds the reference model (model/model.py) for ``inputs.llmy_config()`` with
the synthetic weights (tensors with two or more dimensions stored as bf16, the
rest fp32), saves it the way train/checkpoint.py does ({"model": state_dict,
"config": mapping}), converts it with llmy_cuda/tools/convert_checkpoint.py
into ``tests/golden/tiny_model.llmy`` and records the configuration mapping in
``tests/golden/llmy.npz``.  It also checks that hybrid_llm_b200.llmy_format
writes the same bytes for the same checkpoint.  Nothing at test time reads the
reference.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("LLMY_REFERENCE",
                        Path(__file__).resolve().parents[2].parent / "reference"))
sys.path.insert(0, str(HERE.parents[1]))
sys.path.insert(0, str(HERE))
os.environ.setdefault("LLMY_DISABLE_TRITON", "1")

import torch  # noqa: E402

import inputs  # noqa: E402


def main() -> None:
    if not REF.exists():
        raise SystemExit(f"reference checkout not found at {REF}")
    sys.path.insert(0, str(REF))
    import model.layers.gated_deltanet as gdn_mod
    import model.layers.moe as moe_mod
    gdn_mod._triton_gdn_available = False
    moe_mod._triton_available = False
    from model.config import V6Config
    from model.model import LoopedHybridMoEForCausalLM

    from hybrid_llm_b200 import llmy_format
    from hybrid_llm_b200.weights import synthetic_state_dict

    cfg = inputs.llmy_config()
    mapping = inputs.v6_mapping(cfg)
    model = LoopedHybridMoEForCausalLM(V6Config.from_mapping(mapping)).eval()
    own = dict(model.named_parameters())
    with torch.no_grad():
        for name, t in synthetic_state_dict(cfg, seed=0).items():
            own[name].copy_(t.reshape(own[name].shape))
    sd = {k: (v.bfloat16() if v.dim() >= 2 and v.is_floating_point() else v)
          for k, v in model.state_dict().items()}
    out = HERE / "tiny_model.llmy"
    with tempfile.TemporaryDirectory() as tmp:
        pt = Path(tmp) / "tiny.pt"
        torch.save({"format_version": 1, "model": sd, "config": mapping}, pt)
        subprocess.run([sys.executable, str(REF / "llmy_cuda/tools/convert_checkpoint.py"),
                        str(pt), str(out)], check=True)
        mine = Path(tmp) / "mine.llmy"
        llmy_format.write_llmy(mine, mapping, sd)
        if mine.read_bytes() != out.read_bytes():
            raise SystemExit("llmy_format.write_llmy differs from the reference converter")
    np.savez_compressed(HERE / "llmy.npz", config_json=np.array(json.dumps(mapping)),
                        n_state_tensors=np.array(len(sd)))
    print(f"wrote {out} ({out.stat().st_size} bytes) and llmy.npz")


if __name__ == "__main__":
    main()
