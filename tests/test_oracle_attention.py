"""CPU: attention oracles against the reference's CSA layer and banded SDPA goldens."""
import numpy as np
import pytest

import inputs
from conftest import golden
from oracle import attention


@pytest.mark.parametrize("tag", list(inputs.CSA_CASES))
def test_csa_layer_prefill_matches_reference(tag):
    g = golden("csa")
    c = inputs.csa_case(tag)
    assert g[f"{tag}_checksum"] == inputs.checksum(c["hidden"], *c["p"].values())
    y = attention.csa_layer(c["hidden"], c["p"], c["heads"], c["window"])
    np.testing.assert_allclose(y, g[f"{tag}_out"], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("tag", list(inputs.CSA_CASES))
def test_csa_decode_matches_reference(tag):
    g = golden("csa")
    c = inputs.csa_case(tag)
    p, h, w = c["p"], c["heads"], c["window"]
    seq = c["hidden"].astype(np.float64)
    for i in range(c["steps"].shape[1]):
        seq = np.concatenate([seq, c["steps"][:, i:i + 1]], axis=1)
        win = seq[:, -w:]
        b, L, _ = win.shape
        q = (seq[:, -1] @ p["query"].T).reshape(b, h, -1)
        k = (win @ p["key"].T).reshape(b, L, h, -1)
        v = win @ p["value"].T
        local = attention.csa_local_step(q, k, v)
        y = (local @ p["local_out"].T) @ p["out"].T
        np.testing.assert_allclose(y, g[f"{tag}_step_out"][:, i, 0], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("tag", list(inputs.BAND_CASES))
def test_banded_sdpa_matches_reference(tag):
    g = golden("band")
    c = inputs.band_case(tag)
    assert g[f"{tag}_checksum"] == inputs.checksum(c["q"], c["k"], c["v"])
    y = attention.banded_attention(c["q"], c["k"], c["v"], c["window"])
    np.testing.assert_allclose(y, g[f"{tag}_out"], rtol=1e-4, atol=1e-5)


def test_csa_equals_mean_of_per_head_attention_with_shared_v():
    rng = np.random.default_rng(0)
    q, k = rng.normal(size=(2, 2, 30, 3, 8))
    v = rng.normal(size=(2, 30, 12))
    a = attention.csa_local(q, k, v, 7)
    b = attention.banded_attention(q, k, v[:, :, None, :], 7).mean(axis=2)
    np.testing.assert_allclose(a, b, atol=1e-12)
