"""Layers loaded from a sharded Espalier checkpoint straight onto the GPU, run through the library and checked against
the CPU oracle on the checkpoint's own tensors: the fused q/k/v layer (two launches: int5 4-bit q/k, mcg 2-bit v) and
o (E2M1 by the mul1 marker) within the dense tolerance, every expert matrix's decoded weights bit for bit."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from helpers import LM, bits, f32, floor_err, rel_err, write_checkpoint

from vllm_espalier_b200 import checkpoint as ck
from vllm_espalier_b200 import dense as D
from vllm_espalier_b200.experts import KERNEL_CB, dequant

pytestmark = pytest.mark.gpu


def _oracle(x, mats, want_keys, want):
    return np.concatenate([O.dense_matrix(x, want[k]["esp_trellis"].numpy(), want[k]["suh"].numpy(),
                                          want[k]["svh"].numpy(), m.K, KERNEL_CB[m.cb])
                           for m, k in zip(mats, want_keys)], axis=1)


@pytest.mark.parametrize("M", [1, 8, 32])
def test_checkpoint_layers_vs_oracle(dev, tmp_path, M):
    want = write_checkpoint(tmp_path)
    c = ck.Checkpoint(tmp_path)
    x = torch.randn(M, 256, generator=torch.Generator().manual_seed(M)).bfloat16()
    xf = x.float().numpy()
    for prefix, names in (("language_model.model.layers.3.self_attn.qkv_proj", ("q_proj", "k_proj", "v_proj")),
                          ("language_model.model.layers.3.self_attn.o_proj", ("o_proj",))):
        mats = c.layer(prefix, device=dev)
        assert all(m.trellis.is_cuda for m in mats)
        y = D.Dense(mats).forward(x.to(dev))
        torch.cuda.synchronize()
        ref = _oracle(xf, mats, [f"{LM}.3.self_attn.{n}" for n in names], want)
        e, fl = rel_err(f32(y), ref), floor_err(ref, y.dtype)
        assert e < 1e-2 and e < fl + 2e-3, f"{prefix}: max rel err {e:.3e} (floor {fl:.3e})"


def test_checkpoint_experts_decode_bit_exact(dev, tmp_path):
    want = write_checkpoint(tmp_path)
    ex = ck.Checkpoint(tmp_path).experts("language_model.model.layers.0.mlp.experts", device=dev)
    for e, mats in enumerate(ex):
        for m, p in zip(mats, ck.PROJS):
            T = want[f"{LM}.0.mlp.experts.{e}.{p}"]["esp_trellis"].numpy()
            got = bits(dequant(m.trellis, m.K, m.cb))
            assert np.array_equal(got, O.bits16(O.dequant(T, m.K, KERNEL_CB[m.cb]))), f"expert {e} {p}"
