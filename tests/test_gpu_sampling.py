"""GPU: device sampler vs the oracle (exact tokens for the same uniforms)."""
import numpy as np
import pytest
import torch

import inputs
from conftest import golden
from oracle import sampling

pytestmark = pytest.mark.gpu


def _run(logits, generated, temp, top_k, top_p, rep, uniforms, blocked=None):
    from hybrid_llm_b200 import kernels
    lg = torch.from_numpy(np.ascontiguousarray(logits, dtype=np.float32)).cuda()
    seen = kernels.seen_bitmask(generated, lg.shape[1], "cuda")
    bl = None if blocked is None else torch.tensor(blocked, dtype=torch.int32, device="cuda")
    tok, lp = kernels.sample(lg, temperature=temp, top_k=top_k, top_p=top_p,
                             repetition_penalty=rep, seen=seen, blocked=bl,
                             uniforms=torch.from_numpy(np.asarray(uniforms, np.float32)).cuda(),
                             update_seen=True)
    torch.cuda.synchronize()
    kernels.check_device_status()
    return tok.cpu().numpy(), lp.cpu().numpy(), seen


@pytest.mark.parametrize("tag", list(inputs.SAMPLE_CASES))
def test_sampler_reproduces_reference_tokens(cuda, tag):
    g = golden("sample")
    c = inputs.sample_case(tag)
    tok, lp, _ = _run(c["logits"], c["generated"], c["temp"], c["top_k"], c["top_p"], c["rep"],
                      c["uniforms"])
    np.testing.assert_array_equal(tok, g[f"{tag}_tokens"])
    np.testing.assert_allclose(lp, g[f"{tag}_logprob"], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("b,v", [(1, 32000), (64, 64000), (3, 50)])
@pytest.mark.parametrize("mode", ["greedy", "topk", "topk_topp", "topp", "temp"])
def test_sampler_large_vocab(cuda, b, v, mode):
    cfg = dict(greedy=(0.0, 50, 0.9, 1.1), topk=(0.8, 40, 1.0, 1.1), topk_topp=(0.7, 1000, 0.9, 1.05),
               topp=(1.0, 0, 0.6, 1.0), temp=(1.1, 0, 1.0, 1.3))[mode]
    rng = np.random.default_rng(b + v)
    logits = rng.normal(0, 3.0, (b, v)).astype(np.float32)
    generated = [rng.integers(0, v, 30).tolist() for _ in range(b)]
    uniforms = rng.uniform(0, 1, b).astype(np.float32)
    tok, lp, seen = _run(logits, generated, *cfg, uniforms, blocked=[0, 1, 2])
    ref_tok, ref_lp = sampling.sample_next_token(logits, generated, temp=cfg[0], top_k=cfg[1],
                                                 top_p=cfg[2], rep=cfg[3], uniforms=uniforms,
                                                 blocked=[0, 1, 2])
    np.testing.assert_array_equal(tok, ref_tok)
    np.testing.assert_allclose(lp, ref_lp, rtol=1e-4, atol=1e-4)
    words = seen.cpu().numpy().view(np.uint32)
    for r in range(b):
        assert (words[r, tok[r] // 32] >> (tok[r] % 32)) & 1


def test_sampler_rejects_oversized_top_k(cuda):
    from hybrid_llm_b200 import kernels
    with pytest.raises(RuntimeError, match="not supported"):
        kernels.sample(torch.zeros(1, 5000, device="cuda"), temperature=1.0, top_k=2000, top_p=1.0)
