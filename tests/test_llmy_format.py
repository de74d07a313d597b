"""The reference engine's .llmy checkpoint format against a file written by the
reference's own converter (tests/golden/make_llmy.py)."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import inputs
from hybrid_llm_b200 import llmy_format
from hybrid_llm_b200.config import HybridConfig
from hybrid_llm_b200.weights import synthetic_state_dict

GOLDEN = Path(__file__).resolve().parent / "golden"
FIXTURE = GOLDEN / "tiny_model.llmy"


def _mapping():
    return json.loads(str(np.load(GOLDEN / "llmy.npz")["config_json"]))


def _stored(sd):
    """The checkpoint the fixture was converted from: matrices bf16, the rest fp32."""
    return {k: (v.bfloat16() if v.dim() >= 2 else v) for k, v in sd.items()}


def test_reader_parses_the_converter_output():
    f = llmy_format.read_llmy(FIXTURE)
    try:
        assert f.version == 1
        names = list(f.tensors)
        assert names == sorted(names)
        cfg = inputs.llmy_config()
        assert HybridConfig.from_v6(f.config) == cfg
        gate = f.tensors["recurrent_core.0.moe.experts.gate_proj.weight"]
        assert gate.shape == (cfg.moe_experts, cfg.moe_hidden, cfg.d_model)
        assert gate.dtype == torch.bfloat16
        assert f.tensors["final_norm.weight"].dtype == torch.float32
    finally:
        f.close()


def test_tensors_equal_the_converted_weights():
    cfg = inputs.llmy_config()
    sd = _stored(synthetic_state_dict(cfg, seed=0))
    stacked = llmy_format.stack_experts(sd)
    f = llmy_format.read_llmy(FIXTURE)
    try:
        for name, t in stacked.items():
            got = f.tensors[name]
            assert got.dtype == t.dtype, name
            assert torch.equal(got.reshape(t.shape), t), name
    finally:
        f.close()


def test_writer_reproduces_the_converter_bytes(tmp_path):
    want = FIXTURE.read_bytes()
    f = llmy_format.read_llmy(FIXTURE)
    try:
        out = tmp_path / "a.llmy"
        llmy_format.write_llmy(out, f.config_text, f.tensors)
        assert out.read_bytes() == want
        out2 = tmp_path / "b.llmy"
        llmy_format.write_llmy(out2, _mapping(), f.tensors)   # configuration flattened here
        assert out2.read_bytes() == want
    finally:
        f.close()


def test_config_text_round_trip():
    text = llmy_format.read_llmy(FIXTURE).config_text
    assert llmy_format.flatten_config(_mapping()) == text
    assert llmy_format.flatten_config({"model": _mapping(), "optimizer": {"lr": 1}}) == text
    parsed = llmy_format.parse_config(text)
    assert parsed["recurrent_layout"] == ["csa_moe", "gdn_moe"]
    assert parsed["csa"]["local_window"] == 16 and parsed["mhc"]["enabled"] == 0


@pytest.mark.parametrize("cut", [3, 40, 5000])
def test_truncated_or_foreign_files_are_rejected(tmp_path, cut):
    bad = tmp_path / "bad.llmy"
    bad.write_bytes(FIXTURE.read_bytes()[:cut])
    with pytest.raises((ValueError, struct_error())):
        llmy_format.read_llmy(bad)
    foreign = tmp_path / "foreign.llmy"
    foreign.write_bytes(b"GGUF" + FIXTURE.read_bytes()[4:])
    with pytest.raises(ValueError):
        llmy_format.read_llmy(foreign)


def struct_error():
    import struct
    return struct.error


@pytest.mark.gpu
def test_model_from_llmy_equals_model_from_state_dict(cuda):
    """ModelWeights.from_llmy on the converter's file gives the same model as the
    state dict it was converted from: identical prefill and decode logits."""
    from hybrid_llm_b200.model import LoopedHybridModel
    from hybrid_llm_b200.weights import ModelWeights

    cfg = inputs.llmy_config()
    a = LoopedHybridModel(ModelWeights.from_llmy(FIXTURE, "cuda"))
    b = LoopedHybridModel(ModelWeights.from_state_dict(
        cfg, _stored(synthetic_state_dict(cfg, seed=0)), "cuda"))
    ids = torch.randint(0, cfg.vocab_size, (2, 40), generator=torch.Generator().manual_seed(3))
    oa = a.forward(ids.cuda(), last_logits_only=True)
    ob = b.forward(ids.cuda(), last_logits_only=True)
    assert torch.equal(oa.logits, ob.logits)
    nxt = oa.logits[:, -1].argmax(-1)
    for _ in range(2):
        la = a.decode_step(nxt[:, None], oa.state)
        lb = b.decode_step(nxt[:, None], ob.state)
        assert torch.equal(la, lb)
        nxt = la.float().argmax(-1)


def test_converter_tool_reproduces_the_fixture(tmp_path, capsys):
    """convert_checkpoint on the checkpoint the fixture came from writes the
    reference converter's bytes; its error exits match the tool's."""
    f = llmy_format.read_llmy(FIXTURE)
    try:
        sd = {k: v.clone() for k, v in f.tensors.items()}  # the full state, experts stacked
    finally:
        f.close()
    ckpt = tmp_path / "tiny.pt"
    torch.save({"format_version": 1, "model": sd, "config": _mapping()}, ckpt)
    out = tmp_path / "tiny.llmy"
    assert llmy_format._main(["convert", str(ckpt), str(out)]) == 0
    assert out.read_bytes() == FIXTURE.read_bytes()
    # --keep-fp32 stores float32 copies, --strict rejects the bf16 ones
    out32 = tmp_path / "tiny32.llmy"
    assert llmy_format.convert_checkpoint(ckpt, out32, keep_fp32=True) == 0
    f = llmy_format.read_llmy(out32)
    try:
        assert all(t.dtype == torch.float32 for t in f.tensors.values())
    finally:
        f.close()
    assert llmy_format.convert_checkpoint(ckpt, tmp_path / "x.llmy", strict=True) == 1
    torch.save({"model": dict(sd)}, tmp_path / "nocfg.pt")
    assert llmy_format.convert_checkpoint(tmp_path / "nocfg.pt", tmp_path / "y.llmy") == 1
    assert llmy_format.convert_checkpoint(tmp_path / "missing.pt", tmp_path / "z.llmy") == 1
    err = capsys.readouterr().err
    assert "no 'config' entry" in err and "no such file" in err and "dtype torch.bfloat16" in err
