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
