"""CPU: GDN oracle (recurrence, chunked algebra, layer, decode) against reference goldens."""
import numpy as np
import pytest

import inputs
from conftest import golden
from oracle import gdn


def test_scan_output_matches_reference():
    g = golden("gdn")
    for tag in inputs.GDN_CASES:
        c = inputs.gdn_case(tag)
        p, x = c["p"], c["hidden"].astype(np.float64)
        b, t, _ = x.shape
        h = c["heads"]
        q = gdn.l2norm_heads((x @ p["q_proj"].T).reshape(b, t, h, -1))
        k = gdn.l2norm_heads((x @ p["k_proj"].T).reshape(b, t, h, -1))
        v = (x @ p["v_proj"].T).reshape(b, t, h, -1)
        beta = gdn.sigmoid(x @ p["beta_proj"].T + p["beta_bias"])
        gate = gdn.sigmoid(x @ p["gate_proj"].T).reshape(b, t, h, -1)
        o, _ = gdn.gdn_recurrent(q, k, v, beta, gate, c["reset"], gdn.sigmoid(p["decay_logit"]), c["state"])
        np.testing.assert_allclose(o.reshape(b, t, -1), g[f"{tag}_scan"], rtol=1e-4, atol=2e-5)


def _prefill(tag):
    c = inputs.gdn_case(tag)
    out, s = gdn.gdn_layer(c["hidden"], c["p"], c["state"], c["reset"])
    return c, out, s


@pytest.mark.parametrize("tag", list(inputs.GDN_CASES))
def test_gdn_layer_prefill_matches_reference(tag):
    g = golden("gdn")
    c, out, s = _prefill(tag)
    assert g[f"{tag}_checksum"] == inputs.checksum(c["hidden"], c["state"], *c["p"].values())
    np.testing.assert_allclose(out, g[f"{tag}_out"], rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(s, g[f"{tag}_prefill_state"], rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("tag", list(inputs.GDN_CASES))
def test_gdn_decode_steps_match_reference(tag):
    g = golden("gdn")
    c, _, s = _prefill(tag)
    hist = c["hidden"][:, -3:]
    for i in range(c["steps"].shape[1]):
        x1 = c["steps"][:, i:i + 1]
        y1, s = gdn.gdn_layer(x1, c["p"], s, None, conv_history=hist)
        hist = np.concatenate([hist[:, 1:], x1], axis=1)
        np.testing.assert_allclose(y1, g[f"{tag}_step_out"][:, i], rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(s, g[f"{tag}_step_state"], rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("chunk", [8, 16, 64])
def test_chunked_form_equals_recurrence(chunk):
    rng = np.random.default_rng(chunk)
    b, t, h, k, v = 2, 100, 2, 16, 8
    q = gdn.l2norm_heads(rng.normal(size=(b, t, h, k)))
    kk = gdn.l2norm_heads(rng.normal(size=(b, t, h, k)))
    vv = rng.normal(size=(b, t, h, v))
    beta = rng.uniform(0, 1, (b, t, h))
    gate = rng.uniform(0, 1, (b, t, h, v))
    la = rng.uniform(-0.1, 0, (b, t, h))
    reset = rng.uniform(size=(b, t)) < 0.05
    s0 = rng.normal(size=(b, h, k, v))
    o1, s1 = gdn.gdn_recurrent(q, kk, vv, beta, gate, reset, np.exp(la), s0)
    o2, s2 = gdn.gdn_chunked(q, kk, vv, beta, gate, reset, la, s0, chunk=chunk)
    np.testing.assert_allclose(o2, o1, atol=1e-10)
    np.testing.assert_allclose(s2, s1, atol=1e-10)
