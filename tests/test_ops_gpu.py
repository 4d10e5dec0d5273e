"""The custom-op surface and the prefill paths (the reference's vllm_espalier/ops.py:25-87, experts.py:215-228):
espalier::matmul and espalier::dense over more than 32 rows run in 32-row windows, so every row gets exactly the bits it
gets in decode (windows == rows alone, bit for bit); the gemm prefill branch (dequant + had + cuBLAS fp16) matches the
oracle within its fp16 tolerance; experts.windows over more than 32 rows equals its windows run alone."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import cases as C
import oracle as O
from helpers import f32, floor_err, rel_err

from vllm_espalier_b200 import dense as D
from vllm_espalier_b200 import experts as G
from vllm_espalier_b200 import ops

pytestmark = pytest.mark.gpu
GRID_OF = {1: 0, 3: 1, 6: 3, 7: 4}


class _Mat:
    def __init__(self, T, su, sv, K, cb, dev):
        self.trellis = torch.from_numpy(np.ascontiguousarray(T)).to(dev)
        self.suh = torch.from_numpy(su).to(dev)
        self.svh = torch.from_numpy(sv).to(dev)
        self.K, self.cb = K, GRID_OF[cb]
        self.in_features, self.out_features = T.shape[0] * 16, T.shape[1] * 16


def _mats(name, K, Ns, cb, k2, M, dev):
    mats, xf = C.dense_inputs(name, K, Ns, cb, k2, M, "bf16")
    ms = [_Mat(T, su, sv, k2 // 2, cb, dev) for T, su, sv in mats]
    ref = np.concatenate([O.dense_matrix(xf, T, su, sv, k2 // 2, cb) for T, su, sv in mats], axis=1)
    return ms, xf, ref


def test_matmul_op_windows_equal_rows(dev):
    ms, xf, ref = _mats("op-mm", 256, [256], 6, 8, 70, dev)
    m = ms[0]
    x = torch.from_numpy(xf).to(dev).half()
    y = torch.ops.espalier.matmul(x, m.trellis, m.suh, m.svh, m.K, m.cb)
    rows = torch.cat([torch.ops.espalier.matmul(x[r:r + 1], m.trellis, m.suh, m.svh, m.K, m.cb) for r in range(70)])
    torch.cuda.synchronize()
    assert y.dtype == torch.half and y.shape == (70, 256)
    assert torch.equal(y, rows)
    e, fl = rel_err(f32(y), ref), floor_err(ref, torch.float16)
    assert e < 1e-2 and e < fl + 2e-3, f"max rel err {e:.3e} (floor {fl:.3e})"


def test_dense_op_windows_equal_rows(dev):
    ms, xf, ref = _mats("op-dense", 256, [256, 128], 3, 4, 45, dev)
    d = D.Dense(ms)
    key = ops.register_dense(d)
    x = torch.from_numpy(xf).to(dev).to(torch.bfloat16)
    T, su, sv = [m.trellis for m in ms], [m.suh for m in ms], [m.svh for m in ms]
    y = torch.ops.espalier.dense(x, T, su, sv, key)
    rows = torch.cat([d.forward(x[r:r + 1]) for r in range(45)])
    torch.cuda.synchronize()
    assert torch.equal(y, rows)
    e, fl = rel_err(f32(y), ref), floor_err(ref, torch.bfloat16)
    assert e < 1e-2 and e < fl + 2e-3, f"max rel err {e:.3e} (floor {fl:.3e})"


def test_gemm_prefill_branch(dev, monkeypatch):
    ms, xf, ref = _mats("op-gemm", 512, [256], 7, 8, 64, dev)
    m = ms[0]
    monkeypatch.setattr(ops, "PREFILL", "gemm")            # 64 rows > 32: the op takes the gemm branch
    y = torch.ops.espalier.matmul(torch.from_numpy(xf).to(dev).half(), m.trellis, m.suh, m.svh, m.K, m.cb)
    torch.cuda.synchronize()
    assert y.shape == (64, 256)
    assert rel_err(f32(y), ref) < 1e-2       # cuBLAS fp16 output: the fp16 floor, not a bit pattern


def test_moe_windows_equal_windows_alone(dev):
    experts_np, _, _, _, gate_w = C.moe_inputs()
    mats = [tuple(_Mat(ex[p][0], ex[p][3], ex[p][4], ex[p][1], ex[p][2], dev) for p in ("gate", "up", "down"))
            for ex in experts_np]
    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev).view(torch.bfloat16)  # noqa: E731
    L = G.prepare(mats[:-1], mats[-1], bf(gate_w))
    k, R = C.MOE_K, 40
    s = G.scratch(L, 32, k + 1, dev)
    g = np.random.default_rng(3)
    x = bf(C.activations(("moe-win",), R, C.MOE_D))
    pick = torch.from_numpy(np.stack([g.permutation(C.MOE_E)[:k] for _ in range(R)]).astype(np.int32)).to(dev)
    wts = torch.from_numpy(g.random((R, k)).astype(np.float32)).to(dev)
    out, sh = G.windows(x, pick, wts, L, s)
    a1, s1 = G.routed2(x[:32], pick[:32], wts[:32], L, s)
    a1, s1 = a1.clone(), s1.clone()
    a2, s2 = G.routed2(x[32:], pick[32:], wts[32:], L, s)
    torch.cuda.synchronize()
    assert torch.equal(out[:32], a1) and torch.equal(out[32:], a2)
    assert torch.equal(sh[:32], s1) and torch.equal(sh[32:], s2)
