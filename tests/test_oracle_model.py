"""CPU: the full-model oracle against the reference LoopedHybridMoEForCausalLM goldens."""
import numpy as np

import inputs
from conftest import golden
from hybrid_llm_b200.config import single_block_config
from hybrid_llm_b200.weights import synthetic_state_dict
from oracle.model import OracleModel


def _oracle(cfg):
    sd = synthetic_state_dict(cfg, seed=0)
    return OracleModel(cfg, {k: sd[k] for k in sd})


def test_mini_model_prefill_and_greedy_decode_match_reference():
    g = golden("model")
    m = _oracle(inputs.mini_config())
    logits, state = m.forward(inputs.mini_prompt())
    np.testing.assert_allclose(logits[:, -1], g["mini_prefill_last"], rtol=1e-3, atol=1e-4)
    last = logits[:, -1]
    for i in range(g["mini_tokens"].shape[1]):
        tok = last.argmax(-1)
        np.testing.assert_array_equal(tok, g["mini_tokens"][:, i])
        last, state = m.decode_step(tok, state)
        np.testing.assert_allclose(last, g["mini_step_logits"][:, i], rtol=1e-3, atol=1e-4)


def test_single_block_loop_matches_reference():
    g = golden("model")
    assert g["block_checksum"] == inputs.checksum(inputs.block_hidden())
    m = _oracle(single_block_config())
    out = m.run_stack(inputs.block_hidden(), m.new_state(1))
    np.testing.assert_allclose(out[0, ::4], g["block_out_rows"], rtol=1e-3, atol=1e-4)


def test_package_decode_step_drops_the_loop_output():
    """model/model.py's decode_step returns head(embedding) when all rows are active;
    the standalone sampler copy (the one pinned above) carries the loop output."""
    g = golden("model")
    np.testing.assert_allclose(g["mini_pkg_prefill_last"], g["mini_prefill_last"], rtol=1e-4, atol=1e-5)
    m = _oracle(inputs.mini_config())
    tok = g["mini_tokens"][:, 0]
    emb_only = m.head(m.embed(tok))
    np.testing.assert_allclose(g["mini_pkg_step0_logits"], emb_only, rtol=1e-3, atol=1e-4)
    assert np.abs(g["mini_step_logits"][:, 0] - emb_only).max() > 1e-2


def test_mhc_model_prefill_and_greedy_decode_match_reference():
    """Four hyper-connection streams (model/layers/mhc.py) around every sub-layer."""
    g = golden("mhc")
    np.testing.assert_allclose(g["mhc_prefill_last"], g["mhc_sa_prefill_last"], rtol=1e-5, atol=1e-6)
    m = _oracle(inputs.mhc_config())
    logits, state = m.forward(inputs.mini_prompt())
    np.testing.assert_allclose(logits[:, -1], g["mhc_prefill_last"], rtol=1e-5, atol=1e-5)
    last = logits[:, -1]
    for i in range(g["mhc_tokens"].shape[1]):
        tok = last.argmax(-1)
        np.testing.assert_array_equal(tok, g["mhc_tokens"][:, i])
        last, state = m.decode_step(tok, state)
        np.testing.assert_allclose(last, g["mhc_step_logits"][:, i], rtol=1e-5, atol=1e-5)


def test_mhc_config_conversion():
    import pytest
    from hybrid_llm_b200.config import HybridConfig

    cfg = inputs.mhc_config()
    assert HybridConfig.from_v6(inputs.v6_mapping(cfg)) == cfg
    assert cfg.streams == 4 and inputs.mini_config().streams == 1
    base = inputs.v6_mapping(cfg)
    for key, value in (("shared_across_loops", False),
                       ("preserve_streams_across_loop_boundary", False), ("streams", 3)):
        bad = dict(base, mhc=dict(base["mhc"], **{key: value}))
        with pytest.raises(ValueError):
            HybridConfig.from_v6(bad)
    off = dict(base, mhc=dict(enabled=False, streams=1))
    assert HybridConfig.from_v6(off).mhc_streams == 0


def test_router_context_model_matches_reference():
    """The context-aware router's local-context path (context_router.py:59-133):
    prefill and ten greedy decode steps (the 8-token window wraps)."""
    g = golden("router_ctx")
    np.testing.assert_allclose(g["rc_prefill_last"], g["rc_sa_prefill_last"], rtol=1e-5, atol=1e-6)
    m = _oracle(inputs.router_ctx_config())
    logits, state = m.forward(inputs.mini_prompt())
    np.testing.assert_allclose(logits[:, -1], g["rc_prefill_last"], rtol=1e-5, atol=1e-5)
    last = logits[:, -1]
    for i in range(g["rc_tokens"].shape[1]):
        tok = last.argmax(-1)
        np.testing.assert_array_equal(tok, g["rc_tokens"][:, i])
        last, state = m.decode_step(tok, state)
        np.testing.assert_allclose(last, g["rc_step_logits"][:, i], rtol=1e-5, atol=1e-5)


def test_router_context_config_conversion():
    from hybrid_llm_b200.config import HybridConfig

    cfg = inputs.router_ctx_config()
    assert HybridConfig.from_v6(inputs.v6_mapping(cfg)) == cfg
    assert (cfg.router_context, cfg.router_latent_dim, cfg.router_local_context) == (True, 64, 8)
    # the reference's defaults: context on, latent 256, window 128
    base = inputs.v6_mapping(inputs.mini_config())
    dflt = HybridConfig.from_v6(dict(base, router={}, mla={}))
    assert (dflt.router_context, dflt.router_latent_dim, dflt.router_local_context) == (True, 256, 128)


def test_csa_remote_branch_matches_reference():
    """CSA's remote compressed branch (csa.py:77-131, :208-256;
    compressed_attention.py:85-206): 4-token summaries, top-3 per query and
    head, prefill and eight decode steps (two more summaries complete)."""
    g = golden("csa_remote")
    np.testing.assert_allclose(g["cr_prefill_last"], g["cr_sa_prefill_last"], rtol=1e-5, atol=1e-6)
    m = _oracle(inputs.csa_remote_config())
    logits, state = m.forward(inputs.mini_prompt())
    np.testing.assert_allclose(logits[:, -1], g["cr_prefill_last"], rtol=1e-5, atol=1e-5)
    last = logits[:, -1]
    for i in range(g["cr_tokens"].shape[1]):
        tok = last.argmax(-1)
        np.testing.assert_array_equal(tok, g["cr_tokens"][:, i])
        last, state = m.decode_step(tok, state)
        np.testing.assert_allclose(last, g["cr_step_logits"][:, i], rtol=1e-5, atol=1e-5)


def test_csa_remote_config_conversion():
    from hybrid_llm_b200.config import HybridConfig

    cfg = inputs.csa_remote_config()
    assert HybridConfig.from_v6(inputs.v6_mapping(cfg)) == cfg
    off = inputs.v6_mapping(inputs.mini_config())
    assert off["csa"]["temporal_compression"] == 10 ** 9
    assert HybridConfig.from_v6(off).csa_compression == 0


def test_from_v6_rejects_a_half_precision_gdn_state():
    import pytest
    from hybrid_llm_b200.config import HybridConfig

    base = inputs.v6_mapping(inputs.mini_config())
    HybridConfig.from_v6(dict(base, gdn=dict(base["gdn"], sensitive_state_dtype="fp32")))
    with pytest.raises(ValueError):
        HybridConfig.from_v6(dict(base, gdn=dict(base["gdn"], sensitive_state_dtype="float16")))


def test_shared_experts_match_reference():
    """Shared experts (moe.py:185-198, decode :221-234): every token through
    each, sum / sqrt(n), added to the routed output; prefill and decode."""
    g = golden("shared")
    np.testing.assert_allclose(g["sh_prefill_last"], g["sh_sa_prefill_last"], rtol=1e-5, atol=1e-6)
    m = _oracle(inputs.shared_experts_config())
    logits, state = m.forward(inputs.mini_prompt())
    np.testing.assert_allclose(logits[:, -1], g["sh_prefill_last"], rtol=1e-5, atol=1e-5)
    last = logits[:, -1]
    for i in range(g["sh_tokens"].shape[1]):
        tok = last.argmax(-1)
        np.testing.assert_array_equal(tok, g["sh_tokens"][:, i])
        last, state = m.decode_step(tok, state)
        np.testing.assert_allclose(last, g["sh_step_logits"][:, i], rtol=1e-5, atol=1e-5)


def test_shared_experts_config_and_model_guard():
    import types

    import pytest
    from hybrid_llm_b200.config import HybridConfig
    from hybrid_llm_b200.model import LoopedHybridModel

    cfg = inputs.shared_experts_config()
    assert HybridConfig.from_v6(inputs.v6_mapping(cfg)) == cfg and cfg.moe_shared == 2
    # served on one device; refused under expert parallelism
    with pytest.raises(NotImplementedError):
        LoopedHybridModel(types.SimpleNamespace(cfg=cfg), ep=object())


def test_combined_features_match_reference():
    """mHC (4 streams) + the router's local context + the CSA remote branch +
    shared experts on one model: prefill and six decode steps."""
    g = golden("combined")
    np.testing.assert_allclose(g["cb_prefill_last"], g["cb_sa_prefill_last"], rtol=1e-5, atol=1e-6)
    m = _oracle(inputs.combined_config())
    logits, state = m.forward(inputs.mini_prompt())
    np.testing.assert_allclose(logits[:, -1], g["cb_prefill_last"], rtol=1e-5, atol=1e-5)
    last = logits[:, -1]
    for i in range(g["cb_tokens"].shape[1]):
        tok = last.argmax(-1)
        np.testing.assert_array_equal(tok, g["cb_tokens"][:, i])
        last, state = m.decode_step(tok, state)
        np.testing.assert_allclose(last, g["cb_step_logits"][:, i], rtol=1e-5, atol=1e-5)


def test_loop_memory_matches_reference():
    """The loop memory between loops (loop_memory.py:36-66, model/model.py:608-667
    prefill, :840-891 decode): three loops, prefill and four decode steps."""
    g = golden("loop_mem")
    np.testing.assert_allclose(g["lm_prefill_last"], g["lm_sa_prefill_last"], rtol=1e-5, atol=1e-6)
    cfg = inputs.loop_memory_config()
    m = _oracle(cfg)
    logits, state = m.forward(inputs.mini_prompt())
    np.testing.assert_allclose(logits[:, -1], g["lm_prefill_last"], rtol=1e-5, atol=1e-5)
    last = logits[:, -1]
    for i in range(g["lm_tokens"].shape[1]):
        tok = last.argmax(-1)
        np.testing.assert_array_equal(tok, g["lm_tokens"][:, i])
        last, state = m.decode_step(tok, state)
        np.testing.assert_allclose(last, g["lm_step_logits"][:, i], rtol=1e-5, atol=1e-5)
    # the hook matters: without it the same weights give other logits
    import dataclasses
    off = dataclasses.replace(cfg, loop_memory=False)
    sd = synthetic_state_dict(cfg, seed=0)
    base, _ = OracleModel(off, {k: sd[k] for k in sd}).forward(inputs.mini_prompt())
    moved = np.abs(base[:, -1] - g["lm_prefill_last"]).max() / np.abs(g["lm_prefill_last"]).max()
    assert moved > 0.05, moved


def test_loop_memory_config_conversion():
    import pytest
    from hybrid_llm_b200.config import HybridConfig

    cfg = inputs.loop_memory_config()
    assert HybridConfig.from_v6(inputs.v6_mapping(cfg)) == cfg
    base = inputs.v6_mapping(cfg)
    with pytest.raises(ValueError):
        HybridConfig.from_v6(dict(base, adaptive_loops=dict(enabled=True)))


def test_forced_routes_reproduce_free_routing():
    """OracleModel.forced_routes (the routing-forced full-size parity tests):
    forcing a model's own routes changes nothing; forcing other routes does."""
    cfg = inputs.mini_config()
    m = _oracle(cfg)
    m.route_log = []
    free, st = m.forward(inputs.mini_prompt())
    own = [idx for idx, _ in m.route_log]
    assert len(own) == cfg.num_loops * cfg.n_blocks
    m2 = _oracle(cfg)
    m2.forced_routes = list(own)
    forced, _ = m2.forward(inputs.mini_prompt())
    assert not m2.forced_routes
    np.testing.assert_array_equal(forced, free)
    m3 = _oracle(cfg)
    m3.forced_routes = [np.roll(r, 1, axis=0) for r in own]
    other, _ = m3.forward(inputs.mini_prompt())
    assert np.abs(other - free).max() > 1e-3
