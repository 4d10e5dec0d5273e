"""EspMatrix: one trellis-coded matrix as a checkpoint stores it.

A coded matrix W [in, out] is a packed int16 trellis [in/16, out/16, 16 K] (K bits a weight) plus fp16 sign/scale
vectors suh [in] and svh [out], a `mcg` marker and optionally the codebook markers of codebooks.grid_code. Its
forward is y = H(H(x * suh) @ W) * svh with H the 128-block Hadamard (the reference's matrix.py:19-57), here one
espalier::matmul call.
"""
from __future__ import annotations

import torch

from . import codebooks

REQUIRED = ("esp_trellis", "suh", "svh", "mcg")
SUFFIXES = REQUIRED + ("mul1", "esp_grid")      # every per-matrix tensor a checkpoint may hold


class EspMatrix:
    """trellis / suh / svh (device-movable tensors), in_features, out_features, K (bits a weight) and cb (grid code)."""

    def __init__(self, tensors: dict[str, torch.Tensor]):
        absent = [s for s in REQUIRED if s not in tensors]
        if absent:
            raise ValueError(f"Espalier matrix is missing {absent}")
        t = tensors["esp_trellis"]
        if t.dtype != torch.int16 or t.dim() != 3 or t.shape[2] % 16:
            raise ValueError(f"esp_trellis must be int16 [in/16, out/16, 16K], got {t.dtype} {tuple(t.shape)}")
        self.trellis = t.contiguous()
        self.in_features, self.out_features, self.K = 16 * t.shape[0], 16 * t.shape[1], t.shape[2] // 16
        self.suh = tensors["suh"].to(torch.float16).contiguous()
        self.svh = tensors["svh"].to(torch.float16).contiguous()
        if (self.suh.numel(), self.svh.numel()) != (self.in_features, self.out_features):
            raise ValueError(f"trellis {tuple(t.shape)} is {self.in_features}x{self.out_features} but suh/svh hold "
                             f"{self.suh.numel()}/{self.svh.numel()}")
        self.cb = codebooks.grid_code(tensors)

    def __repr__(self) -> str:
        return (f"EspMatrix({self.in_features}->{self.out_features}, {self.K} bits, "
                f"{codebooks.BY_GRID[self.cb].name})")

    def to(self, device) -> "EspMatrix":
        self.trellis = self.trellis.to(device)
        self.suh = self.suh.to(device)
        self.svh = self.svh.to(device)
        return self

    def weight(self) -> torch.Tensor:
        """W [in, out] fp16, before the Hadamards: the library's decode, bit-identical to the reference's."""
        return dequant(self.trellis, self.K, self.cb)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x [..., in], any float dtype -> [..., out] in x's dtype."""
        return self.forward_with(x, self.trellis, self.suh, self.svh)

    def forward_with(self, x: torch.Tensor, trellis, suh, svh) -> torch.Tensor:
        """forward with the tensors passed in (a vLLM layer's module buffers under torch.compile)."""
        from . import ops  # noqa: F401  (defines torch.ops.espalier)
        lead = x.shape[:-1]
        flat = x.reshape(-1, self.in_features).to(torch.float16).contiguous()
        y = torch.ops.espalier.matmul(flat, trellis, suh, svh, self.K, self.cb)
        return y.reshape(*lead, self.out_features).to(x.dtype)


def dequant(trellis: torch.Tensor, K: int, grid: int) -> torch.Tensor:
    """W [in, out] fp16 of a trellis of K bits a weight and grid code `grid`, through the library's decode kernel."""
    from ._lib import ext
    kin, n = 16 * trellis.shape[0], 16 * trellis.shape[1]
    w = torch.empty((kin, n), dtype=torch.float16, device=trellis.device)
    ext().dequant(trellis.contiguous(), w, 2 * K, codebooks.kernel_id(grid, K))
    return w
