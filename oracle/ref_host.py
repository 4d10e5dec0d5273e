"""The reference plugin's own CUDA kernels, driven the way its Python layer drives them.

TEST AND MEASUREMENT INFRASTRUCTURE ONLY: the reference's extension (its csrc/ built from its sources by
oracle/build_ref.py into oracle/_ref/) is loaded here so that tests/golden/make_golden.py can pin the oracle and
`bench.py --impl reference` can time the reference's kernels beside its CPU path. Nothing of this library's product
imports it.

The launch parameters restate the reference's host code:
  ref_plan          vllm_espalier/dense.py:22-39   (K splits, warps, tiles in flight of a dense launch)
  ref_tile_config   vllm_espalier/experts.py:59-68 (the grouped kernels' tiles)
  RefDense          vllm_espalier/dense.py:53-103  (launch groups, counters and scratch, ext().dense)
  RefMoE            vllm_espalier/experts.py:71-138, 141-177, 206-212, 231-261 (tables, scratch, route, routed2)
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import math
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
SO = HERE / "_ref" / "espalier_ref_ext.so"
KERNEL_CB = {0: 1, 1: 3, 3: 6, 4: 7}       # vllm_espalier/experts.py:34
MAX_ROWS = 32


def available() -> bool:
    return SO.exists()


_EXT = None


def ext():
    global _EXT
    if _EXT is None:
        loader = importlib.machinery.ExtensionFileLoader("espalier_ref_ext", str(SO))
        spec = importlib.util.spec_from_loader("espalier_ref_ext", loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        _EXT = mod
    return _EXT


def ref_plan(K: int, N: int, sms: int):
    nb, kt = N // 128, K // 16
    if nb >= 8 * sms:
        return 1, 4, 1
    if 2 * nb >= 3 * sms and kt % (8 * 2) == 0:
        return 1, 8, 1
    w, sk = 4, 1
    while nb * sk < 2 * sms and kt % (2 * sk * w) == 0 and kt // (2 * sk * w) >= 2:
        sk *= 2
    return sk, w, 1


def ref_tile_config(K: int, N: int, gateup: bool):
    cands = [(4, 4, 4, 2) if gateup else (4, 4, 1, 2), (8, 4, 4, 1) if gateup else (8, 4, 1, 1), (8, 4, 2, 1),
             (8, 4, 1, 1), (4, 4, 2, 2), (4, 4, 1, 2)]
    for nt, w, sk, pf in cands:
        if K % (16 * sk * w) == 0 and N % (16 * nt) == 0:
            return nt, w, sk, pf
    raise ValueError((K, N))


_SCRATCH: dict = {}


def _dense_scratch(dev, z_floats: int, xh_halves: int):
    z, xh = _SCRATCH.get(dev, (None, None))
    if z is None or z.numel() < z_floats:
        z = torch.empty(max(z_floats, 1), dtype=torch.float32, device=dev)
    if xh is None or xh.numel() < xh_halves:
        xh = torch.empty(max(xh_halves, 1), dtype=torch.float16, device=dev)
    _SCRATCH[dev] = (z, xh)
    return z, xh


class RefDense:
    """One dense layer (matrices with trellis, suh, svh, K, cb, in_features, out_features) on the reference kernel."""

    def __init__(self, mats, rot_smem: int = 32 * 1024):
        self.mats = list(mats)
        self.K = self.mats[0].in_features
        self.rot_smem = rot_smem
        self.groups = []
        for i, m in enumerate(self.mats):
            key = (2 * m.K, KERNEL_CB[m.cb])
            if self.groups and self.groups[-1][1:] == key and len(self.groups[-1][0]) < 4:
                self.groups[-1][0].append(i)
            else:
                self.groups.append(([i], *key))
        self.col0, c = [], 0
        for m in self.mats:
            self.col0.append(c)
            c += m.out_features
        self.N = c
        dev = self.mats[0].trellis.device
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self.plans, nbt, z = [], 0, 0
        for idx, _, _ in self.groups:
            n = sum(self.mats[i].out_features for i in idx)
            p = ref_plan(self.K, n, sms)
            self.plans.append(p)
            nbt = max(nbt, n // 128)
            z = max(z, p[0] * MAX_ROWS * n)
        self.counters = torch.zeros(2 * nbt, dtype=torch.int32, device=dev)
        self.dev = dev
        _dense_scratch(dev, z, 4 * MAX_ROWS * self.K)

    def forward(self, x, out=None):
        y = out if out is not None else torch.empty((x.shape[0], self.N), dtype=x.dtype, device=x.device)
        z, xh = _SCRATCH[self.dev]
        e = ext()
        for (idx, k2, cb), (sk, w, pf) in zip(self.groups, self.plans):
            e.dense(x, [self.mats[i].trellis for i in idx], [self.mats[i].suh for i in idx],
                    [self.mats[i].svh for i in idx], [self.col0[i] for i in idx], y, xh, z, self.counters, k2, cb,
                    sk, w, pf, self.rot_smem)
        return y


class RefMoE:
    """One MoE layer (routed experts [(gate, up, down)], a shared expert, its gate weight and the router) on the
    reference's fused-routing sequence: route_group, rot_in, grouped, gateup_epilogue, grouped, down_combine2."""

    def __init__(self, experts, shared, gate_w, gate, rows: int = MAX_ROWS, k: int = 8):
        ents = list(experts) + [tuple(shared)]
        self.E = len(ents)
        self.D, self.I = ents[0][0].in_features, ents[0][0].out_features
        dev = ents[0][0].trellis.device
        self.k, self.rows, self.slots = k, rows, k + 1
        self.gate_w, self.gate = gate_w.reshape(-1).contiguous(), gate

        def tables(j):
            ptr = torch.tensor([m[j].trellis.data_ptr() for m in ents], dtype=torch.int64, device=dev)
            k2 = torch.tensor([2 * m[j].K for m in ents], dtype=torch.int32, device=dev)
            cb = torch.tensor([KERNEL_CB[m[j].cb] for m in ents], dtype=torch.int32, device=dev)
            return ptr, k2, cb, [2 * m[j].K for m in ents]

        def stack(j, attr):
            return torch.stack([getattr(m[j], attr).reshape(-1) for m in ents]).contiguous()

        self.t = [tables(j) for j in range(3)]
        self.suh_g, self.suh_u, self.suh_d = stack(0, "suh"), stack(1, "suh"), stack(2, "suh")
        self.svh_g, self.svh_u, self.svh_d = stack(0, "svh"), stack(1, "svh"), stack(2, "svh")
        self.k2_gu = (min(self.t[0][3] + self.t[1][3]), max(self.t[0][3] + self.t[1][3]))
        self.k2_d = (min(self.t[2][3]), max(self.t[2][3]))
        self.cfg_gu, self.cfg_d = ref_tile_config(self.D, self.I, True), ref_tile_config(self.I, self.D, False)
        P = rows * self.slots
        maxu = min(P, self.E)
        D, I = self.D, self.I
        f = dict(device=dev)
        self.xg = torch.zeros((P, D), dtype=torch.float16, **f)
        self.xu = torch.zeros((P, D), dtype=torch.float16, **f)
        self.xd = torch.zeros((P, I), dtype=torch.float16, **f)
        self.z = torch.zeros((max(2 * self.cfg_gu[2] * I, self.cfg_d[2] * D) * P,), dtype=torch.float32, **f)
        self.y = torch.zeros((P, D), dtype=torch.float32, **f)
        self.counter = torch.zeros(1, dtype=torch.int32, **f)
        self.logits = torch.zeros(rows * self.E, dtype=torch.float32, **f)
        self.pick = torch.zeros(P, dtype=torch.int32, **f)
        self.wts = torch.zeros(P, dtype=torch.float32, **f)
        self.ids = torch.zeros(maxu, dtype=torch.int32, **f)
        self.count = torch.zeros(1, dtype=torch.int32, **f)
        self.members = torch.full((maxu * rows,), -1, dtype=torch.int32, **f)

    def window(self, R: int):
        maxu = min(R * self.slots, self.E)
        return self.ids[:maxu], self.members[:maxu * R].view(maxu, R)

    def route(self, x):
        R = x.shape[0]
        ids, mem = self.window(R)
        n = R * self.slots
        ext().route_group(x, self.gate, self.gate_w, self.k, self.E - 1, self.logits, self.counter, self.pick[:n],
                          self.wts[:n], ids, self.count, mem)

    def forward(self, x, out, out_shared):
        """route() then the reference's routed2(pick=None) sequence."""
        e = ext()
        R = x.shape[0]
        self.route(x)
        ids, mem = self.window(R)
        P = R * self.slots
        pk, wt = self.pick[:P], self.wts[:P]
        (gp, gk, gc, _), (up, uk, uc, _), (dp, dk, dc, _) = self.t
        e.rot_in(x, x.stride(0), pk, self.suh_g, self.suh_u, self.xg, self.xu, R, self.D, self.slots, self.E)
        nt, w, sk, pf = self.cfg_gu
        e.grouped(self.xg, self.xu, gp, up, gk, uk, gc, uc, ids, self.count, mem, self.z, 2, self.D, self.I, P, sk,
                  self.slots, nt, w, pf, self.k2_gu[0], self.k2_gu[1])
        e.gateup_epilogue(self.z, pk, self.svh_g, self.svh_u, self.suh_d, self.xd, R, P, self.I, sk, self.slots,
                          self.E, math.inf, 1)
        nt, w, sk, pf = self.cfg_d
        e.grouped(self.xd, self.xd, dp, dp, dk, dk, dc, dc, ids, self.count, mem, self.z, 1, self.I, self.D, P, sk,
                  self.slots, nt, w, pf, self.k2_d[0], self.k2_d[1])
        e.down_combine2(self.z, pk, self.svh_d, self.y, wt, out, out_shared, R, P, self.D, sk, self.slots, self.E,
                        self.k)
