"""GPU: the looped hybrid stack (prefill, decode, CUDA-graph greedy loop) vs the
reference goldens and the fp64 oracle."""
import numpy as np
import pytest
import torch

import inputs
from conftest import golden

pytestmark = pytest.mark.gpu

# bf16 storage / fp32 accumulation against an fp32 reference
HIDDEN_REL = 2e-2   # max |delta_ours - delta_ref| / max |delta_ref| (residual update)
LOGIT_REL = 3e-2    # max |logits - ref| / max |ref|


def _model(cfg):
    from hybrid_llm_b200.model import LoopedHybridModel
    from hybrid_llm_b200.weights import ModelWeights, synthetic_state_dict
    return LoopedHybridModel(ModelWeights.from_state_dict(cfg, synthetic_state_dict(cfg, seed=0), "cuda"))


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.abs(a - b).max() / np.abs(b).max()


def test_single_block_loop_matches_reference(cuda):
    from hybrid_llm_b200.config import single_block_config
    g = golden("model")
    m = _model(single_block_config())
    x = inputs.block_hidden()
    out = m.run_stack(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    got = out[0, ::4].cpu().numpy() - x[0, ::4]
    ref = g["block_out_rows"] - x[0, ::4]
    assert _rel(got, ref) < HIDDEN_REL, _rel(got, ref)


def _greedy_ok(logits, ref_logits, tokens, ref_tokens):
    """Tokens must match except where the reference's top-2 logits are within tolerance."""
    tol = LOGIT_REL * np.abs(ref_logits).max()
    for r in range(len(tokens)):
        if tokens[r] != ref_tokens[r]:
            top2 = np.sort(ref_logits[r])[-2:]
            assert top2[1] - top2[0] <= tol, (r, tokens[r], ref_tokens[r])


def test_mini_model_prefill_and_greedy_decode(cuda):
    g = golden("model")
    m = _model(inputs.mini_config())
    ids = torch.from_numpy(inputs.mini_prompt()).cuda()
    out = m.forward(ids, last_logits_only=True)
    lg = out.logits[:, -1].float().cpu().numpy()
    assert _rel(lg, g["mini_prefill_last"]) < LOGIT_REL
    state = out.state
    tok = torch.from_numpy(g["mini_tokens"][:, 0]).cuda()
    _greedy_ok(lg, g["mini_prefill_last"], lg.argmax(-1), g["mini_tokens"][:, 0])
    for i in range(g["mini_tokens"].shape[1]):
        lg = m.decode_step(tok, state).float().cpu().numpy()
        assert _rel(lg, g["mini_step_logits"][:, i]) < LOGIT_REL, (i, _rel(lg, g["mini_step_logits"][:, i]))
        if i + 1 < g["mini_tokens"].shape[1]:
            _greedy_ok(lg, g["mini_step_logits"][:, i], lg.argmax(-1), g["mini_tokens"][:, i + 1])
            tok = torch.from_numpy(g["mini_tokens"][:, i + 1]).cuda()  # teacher-force the reference
    assert int(state.positions[0]) == inputs.mini_prompt().shape[1] + g["mini_tokens"].shape[1]


def test_graph_decoder_matches_eager_decode(cuda):
    from hybrid_llm_b200.model import GreedyDecoder
    m = _model(inputs.mini_config())
    ids = torch.from_numpy(inputs.mini_prompt()).cuda()
    outs = []
    for use_graph in (False, True):
        o = m.forward(ids, last_logits_only=True)
        dec = GreedyDecoder(m, o.state, use_graph=use_graph)
        dec.prime(o.logits[:, -1].float().argmax(-1))
        toks = [dec.step().clone() for _ in range(8)]
        outs.append(torch.stack(toks, 1).cpu())
    assert torch.equal(outs[0], outs[1])


def test_decode_equals_prefill_of_extended_sequence(cuda):
    """The reference's own parity check (sample_standalone.py:5474-5527): logits of a
    decode step equal the last-position logits of a prefill over the longer prompt."""
    m = _model(inputs.mini_config())
    ids = torch.from_numpy(inputs.mini_prompt()).cuda()
    o = m.forward(ids[:, :-1], last_logits_only=True)
    step = m.decode_step(ids[:, -1], o.state).float().cpu().numpy()
    full = m.forward(ids, last_logits_only=True).logits[:, -1].float().cpu().numpy()
    assert _rel(step, full) < LOGIT_REL
