"""Checkpoint discovery and loading on CPU (the reference's tests/test_config.py cases against its config.py, plus the
tensor loading of its loaders): which vLLM layers are coded, fused layers, the MTP namespace, vision modules, and
EspMatrix objects read back bit for bit from sharded safetensors files."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch
from safetensors.torch import save_file

from helpers import LM, coded_matrix, write_checkpoint

from vllm_espalier_b200 import checkpoint as ck
from vllm_espalier_b200 import dense as D

KEYS = ([f"{LM}.0.linear_attn.{m}.esp_trellis" for m in ("in_proj_qkv", "in_proj_z", "out_proj")] +
        [f"{LM}.3.self_attn.{m}.esp_trellis" for m in ("q_proj", "k_proj", "v_proj", "o_proj")] +
        [f"{LM}.0.mlp.shared_expert.{m}.esp_trellis" for m in ("gate_proj", "up_proj", "down_proj")] +
        [f"{LM}.0.mlp.experts.7.down_proj.esp_trellis", "lm_head.esp_trellis", "mtp.layers.0.mlp.gate_proj.esp_trellis",
         f"{LM}.0.linear_attn.in_proj_a.weight", "model.visual.blocks.0.attn.qkv.weight"])


def _index(tmp_path, keys):
    (tmp_path / ck.INDEX).write_text(json.dumps({"weight_map": {k: "x.safetensors" for k in keys}}))
    return ck.Checkpoint(tmp_path)


def test_text_key():
    assert ck.text_key("language_model.model.layers.3.self_attn.qkv_proj") == "layers.3.self_attn.qkv_proj"
    assert ck.text_key("language_model.lm_head") == "lm_head"
    assert ck.text_key("visual.blocks.0.attn.qkv") is None
    assert ck.text_key("model.mtp.layers.0.mlp.gate_proj") == "mtp.layers.0.mlp.gate_proj"
    assert ck.text_key("model.embed_tokens") is None


def test_fused_and_plain_layers(tmp_path):
    c = _index(tmp_path, KEYS)
    assert c.is_exl3("language_model.model.layers.3.self_attn.qkv_proj")
    assert c.is_exl3("language_model.model.layers.3.self_attn.o_proj")
    assert c.is_exl3("language_model.model.layers.0.linear_attn.in_proj_qkvz")
    assert c.is_exl3("language_model.model.layers.0.mlp.shared_expert.gate_up_proj")
    assert not c.is_exl3("language_model.model.layers.0.linear_attn.in_proj_ba")
    assert not c.is_exl3("language_model.model.layers.0.mlp.gate")
    assert not c.is_exl3("visual.blocks.0.attn.qkv")
    assert c.is_exl3("language_model.lm_head")
    assert c.experts_exl3("language_model.model.layers.0.mlp.experts")
    assert not c.experts_exl3("language_model.model.layers.1.mlp.experts")
    # the MTP head's layer 0 is not the decoder's layer 0
    assert c.is_exl3("mtp.layers.0.mlp.gate_proj") and not c.is_exl3("model.layers.0.mlp.gate_proj")


def test_partly_coded_fused_layer_is_an_error(tmp_path):
    c = _index(tmp_path, [f"{LM}.3.self_attn.q_proj.esp_trellis"])
    with pytest.raises(ValueError):
        c.is_exl3("language_model.model.layers.3.self_attn.qkv_proj")


def test_quant_config_and_empty_checkpoint(tmp_path):
    ck.check_quant_config({"quant_method": "Espalier"})
    with pytest.raises(ValueError):
        ck.check_quant_config({"quant_method": "gptq"})
    with pytest.raises(ValueError):
        _index(tmp_path, ["model.embed_tokens.weight"])
    with pytest.raises(FileNotFoundError):
        ck.Checkpoint(tmp_path / "missing")


@pytest.fixture
def sharded(tmp_path):
    want = write_checkpoint(tmp_path)
    return ck.Checkpoint(tmp_path), want


def _same(m, t):
    assert torch.equal(m.trellis, t["esp_trellis"])
    assert np.array_equal(m.suh.view(torch.int16).numpy(), t["suh"].view(torch.int16).numpy())
    assert np.array_equal(m.svh.view(torch.int16).numpy(), t["svh"].view(torch.int16).numpy())


def test_load_fused_layer_in_shard_order(sharded):
    c, want = sharded
    q, k, v = c.layer("language_model.model.layers.3.self_attn.qkv_proj")
    for m, name in zip((q, k, v), ("q_proj", "k_proj", "v_proj")):
        _same(m, want[f"{LM}.3.self_attn.{name}"])
    assert (q.K, q.cb, q.in_features, q.out_features) == (4, 3, 256, 256)
    assert (k.out_features, v.K, v.cb) == (128, 2, 0)          # v: no esp_grid, no mul1 -> stock mcg
    (o,) = c.layer("language_model.model.layers.3.self_attn.o_proj")
    assert (o.K, o.cb) == (2, 1)                                 # the mul1 marker -> E2M1 codebook
    with pytest.raises(ValueError):
        c.layer("language_model.model.layers.3.mlp.gate_up_proj")


def test_load_experts(sharded):
    c, want = sharded
    ex = c.experts("language_model.model.layers.0.mlp.experts")
    assert len(ex) == 2
    for e, mats in enumerate(ex):
        for m, p in zip(mats, ck.PROJS):
            _same(m, want[f"{LM}.0.mlp.experts.{e}.{p}"])
    assert [(m.K, m.cb) for m in ex[0]] == [(2, 1), (2, 1), (4, 4)]
    assert [(m.K, m.cb) for m in ex[1]] == [(3, 3), (3, 3), (4, 4)]


def test_missing_expert_matrix_is_an_error(tmp_path):
    keys = [f"{LM}.0.mlp.experts.{e}.{p}.esp_trellis" for e in range(3) for p in ck.PROJS
            if (e, p) != (1, "up_proj")]
    c = _index(tmp_path, keys)
    with pytest.raises(RuntimeError, match="1 expert matrices missing"):
        c.experts("language_model.model.layers.0.mlp.experts")


def test_single_file_checkpoint_and_e4m3(tmp_path):
    gen = torch.Generator().manual_seed(6)
    t = coded_matrix(gen, 128, 128, 4, grid=2)                   # esp_grid 2: E4M3
    save_file({f"lm_head.{s}": v for s, v in t.items()}, str(tmp_path / ck.SINGLE))
    c = ck.Checkpoint(tmp_path)
    (m,) = c.layer("lm_head")
    assert m.cb == 2
    with pytest.raises(NotImplementedError):                     # no decode kernel for E4M3, as in the reference
        D.Dense([m])


def test_pinned_to_the_reference_key_logic(tmp_path):
    """tests/golden/checkpoint_keys.json holds the reference's own text_key / is_exl3 / experts_exl3 answers
    (tests/golden/make_checkpoint_keys.py ran its config.py); this module must give the same for every name."""
    gold = json.loads((Path(__file__).parent / "golden" / "checkpoint_keys.json").read_text())
    c = _index(tmp_path, gold["checkpoint_keys"])
    for name, want in gold["names"].items():
        assert ck.text_key(name) == want["text_key"], name
        if want["is_exl3"] == "error":
            with pytest.raises(ValueError):
                c.is_exl3(name)
        else:
            assert c.is_exl3(name) == want["is_exl3"], name
        assert c.experts_exl3(name) == want["experts_exl3"], name
