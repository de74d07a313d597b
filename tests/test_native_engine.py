"""CPU: the native engine's C API (include/llmy.h) in libllmyb.so.

Every entry point the header declares is exported; the loader parses the
`.llmy` configuration before touching CUDA, so its refusals (files that are
not `.llmy`, configurations the persistent step does not serve) and the
null-handle behaviour are checked here without a GPU; llmy_sample against the
reference sampler's golden vectors.  The forward passes are GPU tests
(test_gpu_native_engine.py)."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

import native_llmy as nl
from hybrid_llm_b200 import _native, llmy_format

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"


def test_header_entry_points_are_exported_and_bound():
    text = (ROOT / "include" / "llmy.h").read_text()
    declared = set(re.findall(r"\b(llmyb?_\w+)\s*\(", text)) - {"llmy_h"}
    assert {"llmy_load", "llmy_decode", "llmy_prefill", "llmy_sample"} <= declared
    handle = C.CDLL(str(_native.LIB_PATH))
    assert [n for n in sorted(declared) if not hasattr(handle, n)] == []
    assert declared == set(nl.SIGNATURES)
    nl.lib()


def _write(path, config: str):
    llmy_format.write_llmy(path, config, {})
    return str(path).encode()


SERVED = GOLDEN / "tiny_model.llmy"


def _served_config() -> str:
    f = llmy_format.read_llmy(SERVED)
    try:
        return f.config_text
    finally:
        f.close()


@pytest.mark.parametrize("change,reason", [
    ("mhc.enabled=1", "hyper-connections"),
    ("router.context_aware=1", "router's context"),
    ("moe.shared_experts=2", "shared experts"),
    ("loop_attnres.enabled=1", "loop memory"),
    ("csa.temporal_compression=4", "remote branch"),
    ("stem_blocks=1", "stem / tail"),
    ("recurrent_layout=csa_moe,hca_moe", "hca_moe"),
    ("gdn.qk_head_dim=128", "64-wide"),
    ("d_model=96", "limits"),
    ("num_loops=x", "expected an integer"),
])
def test_load_refuses_what_the_step_does_not_serve(tmp_path, capfd, change, reason):
    key = change.split("=")[0]
    lines = [ln for ln in _served_config().splitlines() if not ln.startswith(key + "=")]
    path = _write(tmp_path / "m.llmy", "\n".join(sorted(lines + [change])) + "\n")
    assert nl.lib().llmy_load(path) is None
    err = capfd.readouterr().err
    assert "[llmy_load]" in err and reason in err, err


def test_load_reports_missing_and_foreign_files(tmp_path, capfd):
    assert nl.lib().llmy_load(str(tmp_path / "missing.llmy").encode()) is None
    bad = tmp_path / "bad.llmy"
    bad.write_bytes(b"GGUF" + bytes(64))
    assert nl.lib().llmy_load(str(bad).encode()) is None
    err = capfd.readouterr().err
    assert "cannot open" in err and "not an .llmy file" in err


def test_served_configuration_passes_the_parser(capfd):
    """Without a GPU the fixture gets past the configuration checks and fails
    at the first CUDA call."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: the GPU tests load the fixture")
    assert nl.lib().llmy_load(str(SERVED).encode()) is None
    err = capfd.readouterr().err
    assert "[llmy_load]" in err and "served" not in err and "cuda" in err.lower(), err


def test_null_handles_are_harmless(capfd):
    L = nl.lib()
    assert L.llmy_vocab_size(None) == 0 and L.llmy_d_model(None) == 0
    assert L.llmy_num_loops(None) == 0 and L.llmy_max_loops(None) == 0
    assert L.llmy_state_new(None) is None
    assert L.llmy_last_executed_loops(None) == 0
    L.llmy_set_num_loops(None, 3)
    L.llmy_free(None)
    L.llmy_state_free(None)
    L.llmy_state_reset(None)
    L.llmy_decode(None, None, 1, 0, 0, None)
    L.llmy_prefill(None, None, None, 4, None)
    assert L.llmyb_engine_routes(None, None, None, 0) < 0
    err = capfd.readouterr().err
    assert "[llmy_decode]" in err and "[llmy_prefill]" in err


def test_sample_matches_the_reference_sampler():
    z = np.load(GOLDEN / "llmy_sample.npz")
    L = nl.lib()
    for i in range(z["token"].size):
        v, lo = int(z["vocab"][i]), int(z["logit_off"][i])
        ro, nr = int(z["recent_off"][i]), int(z["n_recent"][i])
        logits = np.ascontiguousarray(z["logits"][lo:lo + v], dtype=np.float32)
        recent = np.ascontiguousarray(z["recent"][ro:ro + nr], dtype=np.int32)
        st = C.c_uint64(int(z["state_in"][i]))
        tok = L.llmy_sample(nl.fptr(logits), v, float(z["temperature"][i]), int(z["top_k"][i]),
                            float(z["top_p"][i]), float(z["rep"][i]), nl.iptr(recent), nr,
                            C.byref(st))
        assert (tok, st.value) == (int(z["token"][i]), int(z["state_out"][i])), i
