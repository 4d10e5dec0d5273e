"""Dense Espalier layers in one launch (the reference's vllm_espalier/dense.py): every matrix of a vLLM layer, x in the
model's dtype, output written into each matrix's columns, no casts or cat. Up to 32 rows a call (decode).

All matrices of one launch share K and codebook; a layer that mixes them runs one launch per group into the same
output. The kernel's split of the work depends on the layer's shape alone (stream-K over the GPU's SMs), so a row's
bits never depend on the batch.
"""
from __future__ import annotations

import torch

from ._env import env
from ._lib import ext, lib

MAX_ROWS = 32
KERNEL_CB = {0: 1, 1: 3, 3: 6, 4: 7}
ROT_SMEM = int(env("ESPALIER_DENSE_ROTATION_SMEM", str(32 * 1024)))   # accepted for the reference's switch
_scratch: dict = {}


def scratch(device, z_floats: int, xh_halves: int):
    """Shared scratch, grown while layers are prepared (before any graph capture), never during a forward."""
    s = _scratch.get(device)
    if s is None or s[0].numel() < z_floats or s[1].numel() < xh_halves:
        z = max(z_floats, s[0].numel() if s else 0, 1)
        h = max(xh_halves, s[1].numel() if s else 0, 1)
        s = (torch.empty(z, dtype=torch.float32, device=device), torch.empty(h, dtype=torch.half, device=device))
        _scratch[device] = s
    return s


def plan(K: int, N: int, sms: int) -> tuple[int, int, int]:
    """Kept for the reference's interface (dense.py:22-39): the B200 kernel plans its own stream-K split, so this
    returns the neutral (1, 4, 1). ESPALIER_DENSE_TILE_PLAN is accepted and passed through."""
    forced = env("ESPALIER_DENSE_TILE_PLAN")
    if forced:
        sk, w, pf = (int(v) for v in forced.split(","))
        return sk, w, pf
    return 1, 4, 1


class Dense:
    MAX_ROWS = MAX_ROWS

    def __init__(self, mats, n_out: int | None = None):
        self.mats = list(mats)
        m0 = self.mats[0]
        self.K = m0.in_features
        if any(m.in_features != self.K for m in self.mats):
            raise ValueError("all matrices of a dense layer share their input width")
        self.groups = []                       # launches: (matrix indices, k2, kernel cb)
        for i, m in enumerate(self.mats):
            if m.cb not in KERNEL_CB:   # esp_grid 2 (E4M3) has no decode kernel, in the reference either
                raise NotImplementedError(f"matrix {i}: grid code {m.cb} has no decode kernel")
            key = (2 * m.K, KERNEL_CB[m.cb])
            if self.groups and (self.groups[-1][1], self.groups[-1][2]) == key and len(self.groups[-1][0]) < 4:
                self.groups[-1][0].append(i)
            else:
                self.groups.append(([i], *key))
        self.col0 = []
        c = 0
        for m in self.mats:
            self.col0.append(c)
            c += m.out_features
        self.N = c
        self.n_out = n_out or c
        dev = m0.trellis.device
        self.plans = [plan(self.K, sum(self.mats[i].out_features for i in idx), 0) for idx, _, _ in self.groups]
        nbt_max = max(sum(self.mats[i].out_features for i in idx) // 128 for idx, _, _ in self.groups)
        self.counters = torch.zeros(max(nbt_max, 1), dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            z_bytes = lib().esp_dense_z_bytes(MAX_ROWS)
        xh_bytes = lib().esp_dense_xh_bytes(MAX_ROWS, self.K, 4)
        scratch(dev, z_bytes // 4, xh_bytes // 2)

    def forward(self, x, trellis=None, suh=None, svh=None, out=None):
        """x [M, K] (M <= 32) -> [M, n_out] in x's dtype; trellis/suh/svh lists override the matrices' own tensors
        (module buffers under torch.compile)."""
        M = x.shape[0]
        if M > MAX_ROWS:
            raise ValueError(f"{M} rows: Dense.forward takes at most {MAX_ROWS} (use ops windows)")
        trellis = trellis or [m.trellis for m in self.mats]
        suh = suh or [m.suh for m in self.mats]
        svh = svh or [m.svh for m in self.mats]
        y = out if out is not None else torch.empty((M, self.n_out), dtype=x.dtype, device=x.device)
        if self.n_out > self.N:
            y[:, self.N:].zero_()
        z, xh = scratch(x.device, 0, 0)
        if x.stride(-1) != 1:
            x = x.contiguous()
        for (idx, k2, cb), (sk, w, pf) in zip(self.groups, self.plans):
            ext().dense(x, [trellis[i] for i in idx], [suh[i] for i in idx], [svh[i] for i in idx],
                        [self.col0[i] for i in idx], y, xh, z, self.counters, k2, cb, sk, w, pf, ROT_SMEM)
        return y
