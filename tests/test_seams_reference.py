"""CPU: the hook replacements installed into the reference's own modules.

Where the reference checkout is present (LLMY_REFERENCE, by default the
directory ``reference`` beside this repository; skipped elsewhere, e.g. on
the GPU box): imports model.layers.moe, model.layers.gated_deltanet and
runpod.kernels.triton_banded_attention from it, runs seams.install() on the
real modules, and checks that
* every hook the reference calls now resolves to the replacement, with the
  availability flags its call sites test switched on and the numba fast
  paths that precede the Triton ones (gated_deltanet.py:188-213) switched off;
* every call the reference makes through a hook -- found by parsing the
  modules' source (moe.py:163-167, gated_deltanet.py:184-187, :219-235,
  csa.py:49-53) -- binds to the replacement's signature.
The CUDA results of the replacements are the GPU tests in test_seams.py.
"""
import ast
import inspect
import os
import sys
from pathlib import Path

import pytest

REF = Path(os.environ.get("LLMY_REFERENCE",
                          Path(__file__).resolve().parents[1].parent / "reference"))
HOOKS = {"_triton_moe_dispatch": "triton_moe_dispatch", "_triton_gdn_scan": "triton_gdn_scan",
         "_triton_gdn_step": "triton_gdn_step",
         "triton_banded_local_attention": "triton_banded_local_attention"}

pytestmark = pytest.mark.skipif(not (REF / "model" / "layers" / "moe.py").exists(),
                                reason="reference checkout not present")


@pytest.fixture()
def reference_modules():
    os.environ.setdefault("LLMY_DISABLE_TRITON", "1")
    before = set(sys.modules)
    sys.path.insert(0, str(REF))
    try:
        import importlib
        mods = tuple(importlib.import_module(n) for n in (
            "model.layers.moe", "model.layers.gated_deltanet",
            "runpod.kernels.triton_banded_attention"))
        yield mods
    finally:
        sys.path.remove(str(REF))
        for name in set(sys.modules) - before:
            if name.split(".")[0] in ("model", "runpod"):
                del sys.modules[name]


def _hook_calls(path: Path):
    """(hook name, positional count, keyword names, line) of every call in a file."""
    out = []
    for node in ast.walk(ast.parse(path.read_text())):
        if isinstance(node, ast.Call) and isinstance(node.func, ast.Name) and node.func.id in HOOKS:
            out.append((node.func.id, len(node.args), [k.arg for k in node.keywords], node.lineno))
    return out


def test_install_points_the_reference_hooks_at_the_replacements(reference_modules):
    from hybrid_llm_b200 import seams
    moe, gdn, band = reference_modules
    seams.install(moe, gdn, band)
    assert moe._triton_moe_dispatch is seams.triton_moe_dispatch and moe._triton_available
    assert gdn._triton_gdn_scan is seams.triton_gdn_scan
    assert gdn._triton_gdn_step is seams.triton_gdn_step and gdn._triton_gdn_available
    assert gdn._fused_gdn_scan is None and gdn._fused_gdn_step is None
    assert band.triton_banded_local_attention is seams.triton_banded_local_attention


def test_every_reference_call_site_binds_to_the_replacement(reference_modules):
    from hybrid_llm_b200 import seams
    files = [REF / "model" / "layers" / f for f in ("moe.py", "gated_deltanet.py", "csa.py")]
    calls = [c for f in files for c in _hook_calls(f)]
    assert {c[0] for c in calls} == set(HOOKS), calls
    for name, npos, kws, line in calls:
        sig = inspect.signature(getattr(seams, HOOKS[name]))
        sig.bind(*([None] * npos), **{k: None for k in kws})  # raises TypeError on a mismatch
