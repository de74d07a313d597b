"""Host-side behaviour of RecurrentState (CPU tensors): every table, the
router-latent rings included, takes part in reset, zeroing and the
state_dict round trip."""
import torch

import inputs
from hybrid_llm_b200.state import RecurrentState, state_key


def _filled(cfg, batch=3):
    st = RecurrentState(cfg, batch, "cpu")
    g = torch.Generator().manual_seed(0)
    for table in (st.gdn_states, st.gdn_conv_histories, st.local_k, st.local_v, st.router_latents):
        for t in table.values():
            t.copy_(torch.randn(t.shape, generator=g))
    st.positions.fill_(9)
    return st


def test_router_latent_rings_are_allocated_per_loop_and_block():
    cfg = inputs.router_ctx_config()
    st = RecurrentState(cfg, 2, "cpu")
    assert set(st.router_latents) == {state_key(i, j) for i in range(cfg.num_loops)
                                       for j in range(cfg.n_blocks)}
    t = st.router_latents[state_key(1, 0)]
    assert tuple(t.shape) == (2, cfg.router_local_context, cfg.router_latent_dim)
    assert t.dtype == torch.float32
    assert RecurrentState(inputs.mini_config(), 2, "cpu").router_latents == {}


def test_reset_rows_and_zero_cover_every_table():
    cfg = inputs.router_ctx_config()
    st = _filled(cfg)
    st.reset_rows(torch.tensor([False, True, False]))
    for table in (st.gdn_states, st.gdn_conv_histories, st.router_latents):
        for t in table.values():
            assert not t[1].any() and t[0].any() and t[2].any()
    assert st.positions.tolist() == [9, 0, 9]
    st.zero_()
    for table in (st.gdn_states, st.gdn_conv_histories, st.local_k, st.local_v, st.router_latents):
        assert all(not t.any() for t in table.values())
    assert not st.positions.any()


def test_state_dict_round_trip():
    cfg = inputs.router_ctx_config()
    a = _filled(cfg)
    b = RecurrentState(cfg, 3, "cpu")
    b.load_state_dict(a.state_dict())
    for name in ("gdn_states", "gdn_conv_histories", "local_k", "local_v", "router_latents"):
        ta, tb = getattr(a, name), getattr(b, name)
        assert ta.keys() == tb.keys() and all(torch.equal(ta[k], tb[k]) for k in ta)
    assert torch.equal(a.positions, b.positions)
    assert b.nbytes() == a.nbytes() > 0


def test_state_dict_carries_folded_rings_into_a_fresh_state():
    """A state the persistent step advanced (folded value rings, local_vo)
    restores into a new state that has not created those rings yet."""
    cfg = inputs.router_ctx_config()
    a = _filled(cfg)
    for key, v in a.local_v.items():
        a.local_vo[key] = torch.randn_like(v.float()).to(v.dtype)
    a.folded_rings = True
    b = RecurrentState(cfg, 3, "cpu")
    assert not b.local_vo
    b.load_state_dict(a.state_dict())
    assert b.folded_rings and b.local_vo.keys() == a.local_vo.keys()
    assert all(torch.equal(a.local_vo[k], b.local_vo[k]) for k in a.local_vo)
