"""The vLLM-facing pieces on CPU (skipped where vLLM cannot be imported): the "espalier" quantization config's
checkpoint discovery (the reference's tests/test_config.py cases against its config.py), EspLinearMethod's weight
loading into per-shard EspMatrix objects in vLLM's shard order (the reference's linear.py), EspMoEMethod's per-expert
loading (the reference's moe.py), and the switch salting of vLLM's compile-cache hash."""
from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

from helpers import LM, write_checkpoint

from vllm_espalier_b200 import plugin
from vllm_espalier_b200.matrix import SUFFIXES


@pytest.fixture(scope="module")
def cfg_mod():
    """vLLM is imported only by the tests that run (never under -m gpu, which deselects them all)."""
    pytest.importorskip("vllm")
    from vllm_espalier_b200 import config
    return config


@pytest.fixture(scope="module")
def lin(cfg_mod):
    from vllm_espalier_b200 import linear
    return linear


@pytest.fixture
def cfg(tmp_path, cfg_mod):
    keys = ([f"{LM}.3.self_attn.{m}.esp_trellis" for m in ("q_proj", "k_proj", "v_proj", "o_proj")] +
            [f"{LM}.0.mlp.experts.7.down_proj.esp_trellis", "lm_head.esp_trellis",
             f"{LM}.0.mlp.gate.weight", "model.visual.blocks.0.attn.qkv.weight"])
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {k: "x" for k in keys}}))
    c = cfg_mod.EspalierConfig.from_config({"quant_method": "espalier"})
    c.maybe_update_config(str(tmp_path))
    return c


def test_config_surface(cfg, cfg_mod):
    assert cfg.get_name() == "espalier"
    assert cfg.get_min_capability() == 100
    assert cfg.packed_modules_mapping["qkv_proj"] == ["q_proj", "k_proj", "v_proj"]
    assert cfg_mod.EspalierConfig.override_quantization_method({"quant_method": "espalier"}, None) == "espalier"
    assert cfg_mod.EspalierConfig.override_quantization_method({"quant_method": "awq"}, None) is None
    with pytest.raises(ValueError):
        cfg_mod.EspalierConfig.from_config({"quant_method": "awq"})


def test_config_discovery(cfg, cfg_mod):
    assert cfg.is_exl3("language_model.model.layers.3.self_attn.qkv_proj")
    assert cfg.is_exl3("language_model.model.layers.3.self_attn.o_proj")
    assert cfg.is_exl3("language_model.lm_head")
    assert not cfg.is_exl3("language_model.model.layers.0.mlp.gate")
    assert not cfg.is_exl3("visual.blocks.0.attn.qkv")
    assert cfg.experts_exl3("language_model.model.layers.0.mlp.experts")
    assert cfg_mod.EspalierConfig().is_exl3("language_model.lm_head") is False   # nothing discovered yet


def _load(layer, c, names, order):
    """Feed the checkpoint tensors of `names` through the layer's loaders, shards in `order`."""
    for shard in order:
        base = c.bases[f"layers.3.self_attn.{names[shard]}"]
        for suffix, t in c.tensors(base).items():
            getattr(layer, suffix).weight_loader(getattr(layer, suffix), t, shard)


def test_linear_method_loads_shards_in_vllm_order(tmp_path, monkeypatch, lin):
    from vllm_espalier_b200 import checkpoint as ck
    want = write_checkpoint(tmp_path)
    c = ck.Checkpoint(tmp_path)
    monkeypatch.setattr(lin, "FUSED_DENSE", False)       # the fused layer needs the GPU library; loading does not
    m = lin.EspLinearMethod("language_model.model.layers.3.self_attn.qkv_proj")
    layer = torch.nn.Module()
    m.create_weights(layer, 256, [256, 128, 128], 256, 512, torch.bfloat16)
    assert {n for n, _ in layer.named_parameters()} == set(lin.SUFFIXES)
    _load(layer, c, {"q": "q_proj", "k": "k_proj", "v": "v_proj"}, ["v", "q", "k"])
    m.process_weights_after_loading(layer)
    assert [x.out_features for x in layer.espalier.mats] == [256, 128, 128] and layer.espalier.pad == 0
    for i, name in enumerate(("q_proj", "k_proj", "v_proj")):
        assert torch.equal(getattr(layer, f"esp_trellis_{i}"), want[f"{LM}.3.self_attn.{name}"]["esp_trellis"])
    assert (layer.espalier.mats[2].K, layer.espalier.mats[2].cb) == (2, 0)
    assert layer.espalier.key is None


def test_linear_method_padding_and_errors(tmp_path, monkeypatch, lin):
    from vllm_espalier_b200 import checkpoint as ck
    write_checkpoint(tmp_path)
    c = ck.Checkpoint(tmp_path)
    monkeypatch.setattr(lin, "FUSED_DENSE", False)
    m = lin.EspLinearMethod("language_model.model.layers.3.self_attn.o_proj")
    layer = torch.nn.Module()
    m.create_weights(layer, 256, [384], 256, 384, torch.bfloat16)        # 128 columns of padding
    _load(layer, c, {None: "o_proj"}, [None])
    m.process_weights_after_loading(layer)
    assert layer.espalier.pad == 128
    bad = torch.nn.Module()
    m.create_weights(bad, 512, [256], 512, 256, torch.bfloat16)         # the layer's input width differs
    _load(bad, c, {None: "o_proj"}, [None])
    with pytest.raises(RuntimeError):
        m.process_weights_after_loading(bad)
    head = torch.nn.Module()
    lin.EspLinearMethod("lm_head").create_weights(head, 256, [256], 256, 256, torch.bfloat16)
    lin.EspLinearMethod("lm_head").process_weights_after_loading(head)   # an unloaded drafter head is allowed
    assert head.espalier.mats == [] and head.espalier.key is None
    with pytest.raises(RuntimeError):
        empty = torch.nn.Module()
        m.create_weights(empty, 256, [256], 256, 256, torch.bfloat16)
        m.process_weights_after_loading(empty)


def test_shard_order(lin):
    assert [lin.shard_order(s) for s in (None, "q", "k", "v", (2, 1), 3)] == [0, 0, 1, 2, 1, 3]


def test_switch_salting(monkeypatch):
    class Cfg:
        def compute_hash(self):
            return "0123456789abcdef"
    h = plugin.salted(Cfg.compute_hash)
    monkeypatch.setenv("ESPALIER_PREFILL_MODE", "chunk")
    a = h(Cfg())
    monkeypatch.setenv("ESPALIER_PREFILL_MODE", "gemm")
    b = h(Cfg())
    assert a != b and len(a) == len(b) == 16 and h._esp


def test_register_patches_vllm_once(cfg_mod):
    from vllm.config import VllmConfig
    from vllm.model_executor.layers.quantization import get_quantization_config
    plugin.register()
    first = VllmConfig.compute_hash
    plugin.register()
    assert VllmConfig.compute_hash is first and first._esp
    assert get_quantization_config("espalier") is cfg_mod.EspalierConfig


@pytest.fixture(scope="module")
def moe_mod(cfg_mod):
    from vllm_espalier_b200 import moe
    return moe


def _expert_weights(c, want_prefix):
    """(checkpoint name, tensor) of every expert tensor, as vLLM's loader hands them to the layer."""
    for k in sorted(c.weight_map):
        if k.startswith(want_prefix) and not k.endswith(".weight"):
            base, _, suffix = k.rpartition(".")
            yield k, c.tensors(base)[suffix]


def test_moe_method_loads_experts(tmp_path, moe_mod):
    from vllm_espalier_b200 import checkpoint as ck
    want = write_checkpoint(tmp_path)
    c = ck.Checkpoint(tmp_path)
    m = moe_mod.EspMoEMethod.__new__(moe_mod.EspMoEMethod)       # the config object only feeds vLLM's base class
    assert m.topk_indices_dtype == torch.int32 and m.is_monolithic == moe_mod.ROUTE
    layer = torch.nn.Module()
    m.create_weights(layer, 2, 256, 128, torch.bfloat16)
    names = list(layer.load_weights(_expert_weights(c, f"{LM}.0.mlp.experts.")))
    assert set(names) <= {f"{w}_{s}" for w in ("w13", "w2") for s in SUFFIXES}
    assert "w2_esp_trellis" in names and "w13_esp_grid" in names
    m.process_weights_after_loading(layer)
    assert len(layer.espalier.experts) == 2 and layer.espalier.runner.L is None
    for e, mats in enumerate(layer.espalier.experts):
        for mt, p in zip(mats, ("gate_proj", "up_proj", "down_proj")):
            assert torch.equal(mt.trellis, want[f"{LM}.0.mlp.experts.{e}.{p}"]["esp_trellis"])
    assert [(mt.K, mt.cb) for mt in layer.espalier.experts[1]] == [(3, 3), (3, 3), (4, 4)]


def test_moe_method_errors(tmp_path, moe_mod):
    from vllm_espalier_b200 import checkpoint as ck
    write_checkpoint(tmp_path)
    c = ck.Checkpoint(tmp_path)
    m = moe_mod.EspMoEMethod.__new__(moe_mod.EspMoEMethod)
    layer = torch.nn.Module()
    m.create_weights(layer, 3, 256, 128, torch.bfloat16)               # expert 2 never arrives
    list(layer.load_weights(_expert_weights(c, f"{LM}.0.mlp.experts.")))
    with pytest.raises(RuntimeError, match="3 expert matrices missing"):
        m.process_weights_after_loading(layer)
    bad = torch.nn.Module()
    m.create_weights(bad, 2, 256, 128, torch.bfloat16)
    with pytest.raises(ValueError):
        list(bad.load_weights([("model.layers.0.mlp.experts.gate_up_proj.weight", torch.zeros(1))]))
    gelu = torch.nn.Module()
    m.create_weights(gelu, 2, 256, 128, torch.bfloat16)
    gelu.activation = "gelu"
    list(gelu.load_weights(_expert_weights(c, f"{LM}.0.mlp.experts.")))
    with pytest.raises(NotImplementedError):
        m.process_weights_after_loading(gelu)


def test_loader_keying_pinned_to_the_reference(moe_mod, lin):
    """tests/golden/checkpoint_keys.json holds the reference's own shard_order (linear.py) and expert tensor name
    parsing (moe.py) answers; the methods here key loaded tensors the same way."""
    gold = json.loads((Path(__file__).parent / "golden" / "checkpoint_keys.json").read_text())
    for shard, want in gold["shard_order"]:
        assert lin.shard_order(tuple(shard) if isinstance(shard, list) else shard) == want, shard
    for name, want in gold["expert_names"].items():
        got = moe_mod.parse_expert_tensor(name)
        assert (list(got) if got else None) == want, name
