"""CPU: the sampling oracle against the reference's _sample_next_token goldens."""
import numpy as np
import pytest

import inputs
from conftest import golden
from oracle import sampling


@pytest.mark.parametrize("tag", list(inputs.SAMPLE_CASES))
def test_sampler_matches_reference(tag):
    g = golden("sample")
    c = inputs.sample_case(tag)
    assert g[f"{tag}_checksum"] == inputs.checksum(c["logits"], c["uniforms"])
    for r in range(c["logits"].shape[0]):
        tok, lp, p, _ = sampling.sample_row(c["logits"][r], c["generated"][r], temp=c["temp"],
                                            top_k=c["top_k"], top_p=c["top_p"], rep=c["rep"],
                                            u=float(c["uniforms"][r]))
        assert tok == g[f"{tag}_tokens"][r]
        np.testing.assert_allclose(lp, g[f"{tag}_logprob"][r], rtol=1e-5, atol=1e-5)
        if p is not None:
            np.testing.assert_allclose(p.max(), g[f"{tag}_max_prob"][r], rtol=1e-5)


def test_top_p_keeps_token_that_crosses_threshold():
    logits = np.log(np.array([0.5, 0.3, 0.15, 0.05]))
    # exclusive cumulative: 0, .5, .8, .95 -> top_p=.8 keeps three tokens
    _, _, p, cand = sampling.sample_row(logits, [], temp=1.0, top_k=0, top_p=0.8, rep=1.0, u=0.99)
    assert (p > 0).sum() == 3 and list(cand[:3]) == [0, 1, 2]
