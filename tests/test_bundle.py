"""CPU tests of the quant-bundle reader against the fixture bundle, which the reference's own
cache writer produced from a seeded checkpoint (tests/golden/make_golden.py): the parsed
shape, every quantized linear against the oracle quantizer (pinned to the reference's), the
residual tensors, and the reader's refusals."""
import json
import shutil

import numpy as np
import pytest

from oracle import model as om
from pilm_b200.bundle import LINEARS, NORMS, PREFIX, cache_file_name, read_quant_bundle, read_shape
from tests import _golden as G

VARIANT = "qwen35_w4g128"
BUNDLE = G.GOLDEN / f"bundle_{VARIANT}"


def _cfg():
    z = G.load(f"model_{VARIANT}.npz")
    return G.model_config(z)


def test_shape_from_config():
    cfg, _ = _cfg()
    s = read_shape(BUNDLE)
    assert (s.hidden, s.layers, s.n_heads, s.n_kv_heads, s.head_dim, s.intermediate, s.vocab) == \
        (cfg.hidden, cfg.layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.intermediate, cfg.vocab)
    assert (s.eps, s.rope_theta, s.partial_rotary, s.gated, s.gemma_norm) == \
        (cfg.eps, cfg.rope_theta, cfg.partial_rotary, True, True)


def test_linears_and_residual_match_the_checkpoint():
    cfg, seed = _cfg()
    ck = om.make_checkpoint(cfg, seed)
    host = read_quant_bundle(BUNDLE)
    for li in range(cfg.layers):
        for k, v in LINEARS.items():
            qw, s, kin = host["linears"][f"{PREFIX}layers.{li}.{v}.weight"]
            ref = om.quantize_linear(ck[f"l{li}.{k}"], "w4g128")
            assert kin == ck[f"l{li}.{k}"].shape[1]
            assert np.array_equal(qw.numpy(), ref["qweight"]) and np.array_equal(s.numpy(), ref["scales"])
        for k, v in NORMS.items():
            assert np.array_equal(host["residual"][f"{PREFIX}layers.{li}.{v}.weight"].float().numpy(),
                                  ck[f"l{li}.{k}"].float().numpy())
    qw, s, _ = host["linears"]["lm_head.weight"]
    ref = om.quantize_linear(ck["embed"], "w4g128")
    assert np.array_equal(qw.numpy(), ref["qweight"]) and np.array_equal(s.numpy(), ref["scales"])
    assert np.array_equal(host["residual"][PREFIX + "embed_tokens.weight"].float().numpy(), ck["embed"].float().numpy())


def test_cache_file_names_follow_the_reference_scheme():
    names = {p.name for p in (BUNDLE / "linear_w4a16").iterdir()}
    manifest = json.loads((BUNDLE / "pilm_quant_manifest.json").read_text())
    assert names == {cache_file_name(src) for src in manifest["quantized_linear_sources"]}


def test_reader_refuses_what_it_cannot_run(tmp_path):
    bad = tmp_path / "b"
    shutil.copytree(BUNDLE, bad)
    m = json.loads((bad / "pilm_quant_manifest.json").read_text())
    m["format"] = "something-else"
    (bad / "pilm_quant_manifest.json").write_text(json.dumps(m))
    with pytest.raises(ValueError, match="bundle"):
        read_quant_bundle(bad)
    m["format"] = "pilm-quant-bundle-v1"
    (bad / "pilm_quant_manifest.json").write_text(json.dumps(m))
    c = json.loads((bad / "config.json").read_text())
    c["text_config"]["layer_types"][0] = "linear_attention"
    (bad / "config.json").write_text(json.dumps(c))
    with pytest.raises(ValueError, match="linear-attention"):
        read_quant_bundle(bad)
