"""Test helpers: torch <-> numpy bit views, error measures, and a small sharded checkpoint writer."""
from __future__ import annotations

import json

import numpy as np
import torch
from safetensors.torch import save_file


def to_dev(a: np.ndarray, dev, dtype=None) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t if dtype is None else t.to(dtype)


def bits(t: torch.Tensor) -> np.ndarray:
    """uint16 bit patterns of a 16-bit tensor."""
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def rel_err(y: np.ndarray, ref: np.ndarray) -> float:
    """max |y - ref| / max |ref| (the reference's measure, tests/gpu_dense.py:210-223)."""
    return float(np.abs(y.astype(np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))


def floor_err(ref: np.ndarray, dtype: torch.dtype) -> float:
    """rounding floor of storing ref in dtype, on the same measure."""
    r = torch.from_numpy(np.ascontiguousarray(ref, dtype=np.float32)).to(dtype).float().numpy()
    return rel_err(r, ref)


# ---- a small sharded Espalier checkpoint (safetensors + index), for the checkpoint loader tests ----
LM = "model.language_model.layers"


def coded_matrix(gen, kin, n, bits, grid=None, mul1=False):
    """The checkpoint tensors of one random coded matrix (uniform int16 trellis, +-1 suh, small positive svh)."""
    t = {"esp_trellis": torch.randint(-32768, 32768, (kin // 16, n // 16, 16 * bits), dtype=torch.int16,
                                      generator=gen),
         "suh": (torch.randint(0, 2, (kin,), generator=gen) * 2 - 1).half(),
         "svh": (torch.rand(n, generator=gen) / 64).half(),
         "mcg": torch.zeros(1, dtype=torch.int32)}
    if grid is not None:
        t["esp_grid"] = torch.tensor([grid], dtype=torch.int32)
    if mul1:
        t["mul1"] = torch.zeros(1, dtype=torch.int32)
    return t


def write_checkpoint(path):
    """Two shards: layer 3's q/k/v/o (int5, 4 bits; v stock mcg 2 bits, o with the mul1 marker) and two experts of
    layer 0 (E2M1 2-bit, int5 3-bit, int6 4-bit down), with an index."""
    gen = torch.Generator().manual_seed(5)
    a, b = {}, {}
    want = {}
    for name, (kin, n, bits, grid, mul1) in {
            f"{LM}.3.self_attn.q_proj": (256, 256, 4, 3, False), f"{LM}.3.self_attn.k_proj": (256, 128, 4, 3, False),
            f"{LM}.3.self_attn.v_proj": (256, 128, 2, None, False), f"{LM}.3.self_attn.o_proj": (256, 256, 2, None, True)
    }.items():
        t = coded_matrix(gen, kin, n, bits, grid, mul1)
        want[name] = t
        a.update({f"{name}.{s}": v for s, v in t.items()})
    for e, (grid, bits) in enumerate([(1, 2), (3, 3)]):
        for p, (kin, n) in zip(("gate_proj", "up_proj", "down_proj"), [(256, 128), (256, 128), (128, 256)]):
            name = f"{LM}.0.mlp.experts.{e}.{p}"
            t = coded_matrix(gen, kin, n, 4 if p == "down_proj" else bits, 4 if p == "down_proj" else grid)
            want[name] = t
            b.update({f"{name}.{s}": v for s, v in t.items()})
    save_file(a, str(path / "model-00001-of-00002.safetensors"))
    save_file(b, str(path / "model-00002-of-00002.safetensors"))
    wm = {k: "model-00001-of-00002.safetensors" for k in a} | {k: "model-00002-of-00002.safetensors" for k in b}
    (path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": wm}))
    return want
