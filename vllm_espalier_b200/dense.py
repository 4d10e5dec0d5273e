"""Dense coded layers: every matrix of one vLLM layer (q/k/v, in_proj_qkv/z, o, the LM head) decoded and multiplied in
as few launches of the fused dense kernel (esp_dense) as the matrices' codebooks allow, x and y in the model's dtype,
each matrix writing its own columns of y. Up to 32 rows a call (decode); ops.py runs more rows in 32-row windows.

Surface kept from the reference (vllm_espalier/dense.py): Dense(mats, n_out).forward(x, trellis, suh, svh, out) and
MAX_ROWS. Everything under it is this library's:

  * launches   the layer's matrices are grouped by (bits, codebook) over the whole layer, not only in adjacent runs (a
               launch takes up to 4 matrices of one kind; their columns need not be contiguous in y);
  * tables     each launch's C-ABI matrix table (esp_matrix_t[]) is built and checked once, when the layer is built;
               a forward with other tensors of the same shapes (module buffers under torch.compile) refills it;
  * workspace  the kernel's scratch (rotated activations, split-K partial sums, arrival counters) is one set per
               device shared by every layer, sized while layers are built so a forward never allocates (CUDA graphs).

The kernel's work split depends on the layer's shape and the GPU's SM count only, so a row's bits never depend on the
other rows of the call.
"""
from __future__ import annotations

import torch

from . import codebooks
from ._lib import DTYPE, check, esp_matrix_t, lib, stream_ptr

MAX_ROWS = 32
MAX_PER_LAUNCH = 4


class Workspace:
    """The dense kernel's scratch on one device: xh fp16, z (tagged partial sums, 8-byte words, zero on entry and left
    zero), counters int32 (zero)."""

    def __init__(self, device: torch.device):
        self.device = device
        self.xh = torch.empty(0, dtype=torch.float16, device=device)
        self.z = torch.empty(0, dtype=torch.float32, device=device)
        self.counters = torch.zeros(0, dtype=torch.int32, device=device)

    def reserve(self, xh_bytes: int, z_bytes: int, blocks: int) -> "Workspace":
        if self.xh.numel() * 2 < xh_bytes:
            self.xh = self._new(-(-xh_bytes // 2), torch.float16, zero=False)
        if self.z.numel() * 4 < z_bytes:
            self.z = self._new(-(-z_bytes // 4), torch.float32, zero=True)
        if self.counters.numel() < blocks:
            self.counters = self._new(blocks, torch.int32, zero=True)
        return self

    def _new(self, n: int, dtype, zero: bool) -> torch.Tensor:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("the dense workspace must grow before graph capture: build the layer first")
        return (torch.zeros if zero else torch.empty)(n, dtype=dtype, device=self.device)


_WORKSPACES: dict[torch.device, Workspace] = {}


def workspace(device) -> Workspace:
    device = torch.device(device)
    if device.index is None:
        device = torch.device(device.type, torch.cuda.current_device())
    ws = _WORKSPACES.get(device)
    if ws is None:
        ws = _WORKSPACES[device] = Workspace(device)
    return ws


class _Launch:
    """One esp_dense call: matrices `members` of the layer (one width and codebook), with their C table."""

    def __init__(self, members: list[int], k2: int, cb: int, mats, cols: list[int]):
        self.members, self.k2, self.cb = members, k2, cb
        self.table = (esp_matrix_t * len(members))()
        self.cols = [cols[i] for i in members]
        self.shapes = [(mats[i].in_features, mats[i].out_features) for i in members]
        self.bound: tuple = ()
        self.own = ([mats[i].trellis for i in members], [mats[i].suh for i in members], [mats[i].svh for i in members])
        self.fill(*self.own)
        self.own_key = self.bound          # the table holds the matrices' own tensors while bound is this tuple

    def fill(self, trellis, suh, svh):
        key = tuple(t.data_ptr() for t in (*trellis, *suh, *svh))
        if key == self.bound:
            return
        for j, (t, su, sv, (kin, n)) in enumerate(zip(trellis, suh, svh, self.shapes)):
            if not (t.is_cuda and t.dtype == torch.int16 and t.is_contiguous() and t.shape[0] * 16 == kin
                    and t.shape[1] * 16 == n and t.shape[2] == 8 * self.k2):
                raise ValueError(f"matrix {self.members[j]}: trellis must be contiguous int16 [{kin // 16}, "
                                 f"{n // 16}, {8 * self.k2}] on the GPU")
            for v, size, name in ((su, kin, "suh"), (sv, n, "svh")):
                if not (v.is_cuda and v.dtype == torch.float16 and v.is_contiguous() and v.numel() == size):
                    raise ValueError(f"matrix {self.members[j]}: {name} must be contiguous fp16 [{size}]")
            self.table[j] = esp_matrix_t(t.data_ptr(), su.data_ptr(), sv.data_ptr(), n, self.cols[j])
        self.bound = key


class Dense:
    """The matrices of one layer (EspMatrix-like: trellis, suh, svh, K, cb, in_features, out_features), their outputs
    side by side in the given order; n_out > the summed widths leaves zero columns after them (the head's padding)."""

    MAX_ROWS = MAX_ROWS

    def __init__(self, mats, n_out: int | None = None):
        self.mats = list(mats)
        if not self.mats:
            raise ValueError("a dense layer needs at least one matrix")
        self.K = self.mats[0].in_features
        if any(m.in_features != self.K for m in self.mats):
            raise ValueError("the matrices of one dense layer share their input width")
        cols = [0]
        for m in self.mats:
            cols.append(cols[-1] + m.out_features)
        self.col0, self.N = cols[:-1], cols[-1]
        self.n_out = n_out or self.N
        if self.n_out < self.N:
            raise ValueError(f"n_out {self.n_out} is below the matrices' {self.N} columns")
        kinds: dict[tuple[int, int], list[int]] = {}
        for i, m in enumerate(self.mats):
            kinds.setdefault((2 * m.K, codebooks.kernel_id(m.cb, m.K, f"matrix {i}")), []).append(i)
        self.launches = [_Launch(idx[a:a + MAX_PER_LAUNCH], k2, cb, self.mats, self.col0)
                         for (k2, cb), idx in kinds.items() for a in range(0, len(idx), MAX_PER_LAUNCH)]
        dev = self.mats[0].trellis.device
        with torch.cuda.device(dev):
            z = lib().esp_dense_z_bytes(MAX_ROWS)
        xh = lib().esp_dense_xh_bytes(MAX_ROWS, self.K, MAX_PER_LAUNCH)
        blocks = max(sum(self.mats[i].out_features for i in ln.members) // 128 for ln in self.launches)
        self.ws = workspace(dev).reserve(xh, z, blocks)

    def forward(self, x: torch.Tensor, trellis=None, suh=None, svh=None, out: torch.Tensor | None = None):
        """x [M, K] (M <= 32, fp16/bf16/fp32) -> [M, n_out] in x's dtype. trellis / suh / svh: per-matrix tensors to
        use instead of the matrices' own (same shapes)."""
        if x.dim() != 2 or x.shape[1] != self.K or not x.is_cuda or x.dtype not in DTYPE:
            raise ValueError(f"x must be a CUDA fp16/bf16/fp32 [M, {self.K}] tensor, got {x.dtype} {tuple(x.shape)}")
        M = x.shape[0]
        if M > MAX_ROWS:
            raise ValueError(f"{M} rows: Dense.forward takes at most {MAX_ROWS} (ops.py runs windows)")
        if x.stride(1) != 1:
            x = x.contiguous()
        y = out if out is not None else torch.empty((M, self.n_out), dtype=x.dtype, device=x.device)
        if y.shape != (M, self.n_out) or y.stride(1) != 1 or y.dtype not in DTYPE:
            raise ValueError(f"out must be fp16/bf16/fp32 [{M}, {self.n_out}] with unit column stride")
        if self.n_out > self.N:
            y[:, self.N:].zero_()
        if M == 0:
            return y
        ws, stream = self.ws, stream_ptr(x.device)
        given = trellis is not None or suh is not None or svh is not None
        for ln in self.launches:
            if given:
                ln.fill(*(ln.own[q] if g is None else [g[i] for i in ln.members]
                          for q, g in enumerate((trellis, suh, svh))))
            elif ln.bound is not ln.own_key:
                ln.fill(*ln.own)
                ln.own_key = ln.bound
            check(lib().esp_dense(x.data_ptr(), DTYPE[x.dtype], x.stride(0), M, self.K, ln.table, len(ln.members),
                                  ln.k2, ln.cb, y.data_ptr(), DTYPE[y.dtype], y.stride(0), ws.xh.data_ptr(),
                                  ws.xh.numel() * 2, ws.z.data_ptr(), ws.z.numel() * 4, ws.counters.data_ptr(),
                                  ws.counters.numel(), stream))
        return y

    __call__ = forward
