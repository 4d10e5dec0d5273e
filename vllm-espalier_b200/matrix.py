"""One Espalier matrix: its checkpoint tensors and its forward (the reference's vllm_espalier/matrix.py:19-57).

Tensors per matrix (checkpoint suffixes): esp_trellis (int16 [in/16, out/16, 16K]), suh (fp16 [in]), svh (fp16 [out]),
mcg (marker), and optionally mul1 or esp_grid (int32 code: 1 E2M1, 2 E4M3, 3 int5, 4 int6). Codebook: esp_grid's code
if present, else 1 if mul1 is present, else 0 (stock mcg).

forward(x) = H(H(x * suh) @ W) * svh through the espalier::matmul custom op.
"""
from __future__ import annotations

import torch

SUFFIXES = ("esp_trellis", "suh", "svh", "mcg", "mul1", "esp_grid")


class EspMatrix:
    def __init__(self, tensors: dict[str, torch.Tensor]):
        missing = [s for s in ("esp_trellis", "suh", "svh", "mcg") if s not in tensors]
        if missing:
            raise ValueError(f"Espalier matrix is missing {missing}")
        self.trellis = tensors["esp_trellis"].contiguous()
        if self.trellis.dtype != torch.int16 or self.trellis.dim() != 3:
            raise ValueError(f"esp_trellis must be int16 [in/16, out/16, 16K], got {tuple(self.trellis.shape)}")
        self.suh = tensors["suh"].half().contiguous()
        self.svh = tensors["svh"].half().contiguous()
        self.in_features = self.suh.numel()
        self.out_features = self.svh.numel()
        self.K = self.trellis.shape[-1] // 16
        if self.trellis.shape[0] * 16 != self.in_features or self.trellis.shape[1] * 16 != self.out_features:
            raise ValueError(f"trellis {tuple(self.trellis.shape)} does not match suh/svh {self.in_features}x"
                             f"{self.out_features}")
        if "esp_grid" in tensors:
            self.cb = int(tensors["esp_grid"].flatten()[0].item())
            if self.cb not in (1, 2, 3, 4):
                raise ValueError(f"esp_grid code {self.cb}")
        else:
            self.cb = 1 if "mul1" in tensors else 0

    def to(self, device):
        self.trellis, self.suh, self.svh = (t.to(device) for t in (self.trellis, self.suh, self.svh))
        return self

    def weight(self) -> torch.Tensor:
        """W [in, out] fp16 (before the Hadamards), from the trellis decode kernel."""
        from .experts import dequant
        return dequant(self.trellis, self.K, self.cb)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x [..., in] (any float dtype) -> [..., out] in x's dtype."""
        return self.forward_with(x, self.trellis, self.suh, self.svh)

    def forward_with(self, x, trellis, suh, svh) -> torch.Tensor:
        from . import ops  # noqa: F401  (registers the custom ops)
        shape = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features).half().contiguous()
        y = torch.ops.espalier.matmul(x2, trellis, suh, svh, self.K, self.cb)
        return y.view(*shape, self.out_features).to(x.dtype)
