"""The vLLM layer methods' forward on the GPU, outside a vLLM model (skipped where vLLM cannot be imported): a coded
q/k/v layer loaded through EspLinearMethod's loaders and run by its apply() equals dense.Dense on the same matrices bit
for bit, and a coded expert layer loaded through EspMoEMethod and run by its apply() with vLLM-style top-k ids equals
experts.routed2 on the same experts bit for bit."""
from __future__ import annotations

import pytest
import torch

from helpers import LM, write_checkpoint

from vllm_espalier_b200 import checkpoint as ck

pytestmark = pytest.mark.gpu


def test_linear_method_apply_equals_dense(dev, tmp_path):
    pytest.importorskip("vllm")
    from vllm_espalier_b200 import dense as D
    from vllm_espalier_b200 import linear as lin
    write_checkpoint(tmp_path)
    c = ck.Checkpoint(tmp_path)
    m = lin.EspLinearMethod("language_model.model.layers.3.self_attn.qkv_proj")
    layer = torch.nn.Module()
    with torch.device(dev):                                    # vLLM creates parameters on the GPU
        m.create_weights(layer, 256, [256, 128, 128], 256, 512, torch.bfloat16)
    for shard, name in (("k", "k_proj"), ("q", "q_proj"), ("v", "v_proj")):
        for suffix, t in c.tensors(c.bases[f"layers.3.self_attn.{name}"]).items():
            getattr(layer, suffix).weight_loader(getattr(layer, suffix), t, shard)
    m.process_weights_after_loading(layer)
    assert layer.espalier.key is not None
    x = torch.randn(3, 5, 256, generator=torch.Generator().manual_seed(1)).bfloat16().to(dev)
    y = m.apply(layer, x)
    want = D.Dense(c.layer("language_model.model.layers.3.self_attn.qkv_proj", device=dev)).forward(x.reshape(15, 256))
    torch.cuda.synchronize()
    assert y.shape == (3, 5, 512) and torch.equal(y.reshape(15, 512), want)


def test_moe_method_apply_equals_routed2(dev, tmp_path):
    pytest.importorskip("vllm")
    from vllm_espalier_b200 import experts as G
    from vllm_espalier_b200 import moe
    write_checkpoint(tmp_path)
    c = ck.Checkpoint(tmp_path)
    m = moe.EspMoEMethod.__new__(moe.EspMoEMethod)
    layer = torch.nn.Module()
    with torch.device(dev):
        m.create_weights(layer, 2, 256, 128, torch.bfloat16)
    names = [k for k in sorted(c.weight_map) if k.startswith(f"{LM}.0.mlp.experts.")]
    list(layer.load_weights((k, c.tensors(k.rpartition(".")[0])[k.rpartition(".")[2]]) for k in names))
    m.process_weights_after_loading(layer)
    g = torch.Generator().manual_seed(2)
    x = torch.randn(5, 256, generator=g).bfloat16().to(dev)
    ids = torch.stack([torch.randperm(2, generator=g) for _ in range(5)]).to(torch.int32).to(dev)
    w = torch.softmax(torch.randn(5, 2, generator=g), -1).to(dev)
    got = m.apply(layer, x, w, ids)
    L = G.prepare(c.experts("language_model.model.layers.0.mlp.experts", device=dev))
    s = G.scratch(L, 32, 2, dev)
    want, _ = G.routed2(x, ids, w, L, s)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
