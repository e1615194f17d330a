"""Checkpoint reading (ParseCheckpoint / ApplyParams, Brain/Checkpoint/CheckpointReader.ts) on the host.

The reference's checkpoint tests (Tests/Checkpoint.Test.ts) are round trips through its own writer; here
the writer's byte formats are pinned by known answers (base64 of f64, JSON.stringify numbers, the
sha256 payload), the tensor list against the library's parameter layout, and the reader's refusals by
corrupting a checkpoint.
"""
import hashlib
import json

import numpy as np
import pytest

from tests.helpers import ARCHS, pkg

ck = pkg.checkpoint


@pytest.mark.parametrize("x,want", [(1e-5, "0.00001"), (3e-4, "0.0003"), (0.9, "0.9"), (5000.0, "5000"),
                                    (1e21, "1e+21"), (1e-7, "1e-7"), (2.75, "2.75"), (-0.5, "-0.5"),
                                    (1.5e-10, "1.5e-10"), (100, "100"), (0.1 + 0.2, "0.30000000000000004")])
def test_js_number_formatting(x, want):
    assert ck.js_number(x) == want


def test_js_stringify_and_float64_encoding_known_answers():
    cfg = {"Model": {"EmbedDim": 8, "LayerNormEps": 1e-5, "PositionScheme": "Rope", "WeightTying": True},
           "Data": {"Files": ["a\"b", "c\\d"], "Max": None}}
    assert ck.js_stringify(cfg) == ('{"Model":{"EmbedDim":8,"LayerNormEps":0.00001,"PositionScheme":"Rope",'
                                    '"WeightTying":true},"Data":{"Files":["a\\"b","c\\\\d"],"Max":null}}')
    assert ck.encode_float64(np.array([1.0, 2.0])) == "AAAAAAAA8D8AAAAAAAAAQA=="
    assert ck.encode_float64(np.array([1.0], np.float32)) == "AAAAAAAA8D8="  # f32 widened to f64
    assert ck.decode_float64("AAAAAAAA8D8AAAAAAAAAQA==").tolist() == [1.0, 2.0]
    params = [{"Rows": 1, "Cols": 2, "Data": "AAAAAAAA8D8AAAAAAAAAQA=="}]
    opt = {"M": ["AAAAAAAA8D8="], "V": [], "StepCount": 3}
    want = hashlib.sha256(("1x2:AAAAAAAA8D8AAAAAAAAAQA==" + "AAAAAAAA8D8=" + "3" +
                           '{"Model":{"EmbedDim":8}}').encode()).hexdigest()
    assert ck.checksum_payload(params, opt, {"Model": {"EmbedDim": 8}}) == want


def _config(cfg):
    m = {"EmbedDim": cfg.embed_dim, "NumLayers": cfg.num_layers, "NumHeads": cfg.num_heads,
         "BlockSize": cfg.block_size, "VocabSize": cfg.vocab_size, "MlpRatio": cfg.mlp_hidden / cfg.embed_dim,
         "LayerNormEps": cfg.layer_norm_eps, "Dropout": 0, "WeightTying": cfg.weight_tying, "InitScale": 0.02,
         "UseScaledResidualInit": True, "PositionScheme": cfg.position_scheme, "NormKind": cfg.norm_kind,
         "MlpKind": cfg.mlp_kind}
    if cfg.kv_heads is not None:
        m["KvHeads"] = cfg.kv_heads
    return {"Model": m, "Optimizer": {"Kind": "AdamW", "LearningRate": 3e-4}, "Training": {"Seed": 1}}


@pytest.mark.parametrize("label,arch", ARCHS, ids=[a[0] for a in ARCHS])
def test_tensor_list_matches_parameter_layout_and_round_trips(label, arch):
    cfg = pkg.ModelConfig(**arch)
    shapes = ck.param_shapes(cfg)
    assert sum(r * c for r, c in shapes) == pkg.decode.param_count(cfg)
    p = pkg.init_params(cfg, 3)
    text = json.dumps(ck.build_checkpoint(_config(cfg), p, cfg))
    parsed = ck.parse_checkpoint(text)
    cfg2 = ck.model_config_from(parsed["Config"])
    assert cfg2 == cfg
    got = ck.checkpoint_params(parsed, cfg2)
    assert got.dtype == np.float64 and np.array_equal(got, p.astype(np.float64))


def test_microchat_config_maps_to_the_bench_shape():
    cfg = pkg.configs.MICROCHAT.model
    assert ck.model_config_from(_config(cfg)) == cfg


def test_reader_refuses_corrupt_or_mismatched_checkpoints():
    cfg = pkg.ModelConfig(**ARCHS[2][1])
    p = pkg.init_params(cfg, 3)
    good = ck.build_checkpoint(_config(cfg), p, cfg)
    bad = json.loads(json.dumps(good))
    data = bytearray(ck.base64.b64decode(bad["Params"][3]["Data"]))
    data[5] ^= 1
    bad["Params"][3]["Data"] = ck.base64.b64encode(bytes(data)).decode()
    with pytest.raises(ck.CheckpointError, match="checksum mismatch"):
        ck.parse_checkpoint(json.dumps(bad))
    with pytest.raises(ck.CheckpointError, match="format version"):
        ck.parse_checkpoint(json.dumps(dict(good, FormatVersion=2)))
    # without a checksum the reader still catches truncation and shape drift (ApplyParams)
    trunc = json.loads(json.dumps(good))
    del trunc["Checksum"]
    trunc["Params"][0]["Data"] = ck.encode_float64(np.zeros(3))
    with pytest.raises(ck.CheckpointError, match="payload length"):
        ck.checkpoint_params(ck.parse_checkpoint(json.dumps(trunc)), cfg)
    other = pkg.ModelConfig(**dict(ARCHS[2][1], embed_dim=32))
    with pytest.raises(ck.CheckpointError, match="architecture mismatch"):
        ck.checkpoint_params(good, other)
    shape = json.loads(json.dumps(good))
    shape["Params"][1]["Rows"] = 2
    with pytest.raises(ck.CheckpointError, match="tensor 1 shape"):
        ck.checkpoint_params(shape, cfg)
