"""Routed experts (the reference's vllm_espalier/experts.py): grouped MoE pipeline, fused routing and the weight
decode. This module currently provides the weight decode; the grouped pipeline lives in moe kernels of the library."""
from __future__ import annotations

import torch

from ._lib import ext

# Espalier grid code (EspMatrix.cb) -> the kernels' codebook id (1 mcg, 3 E2M1, 6 int5, 7 int6)
KERNEL_CB = {0: 1, 1: 3, 3: 6, 4: 7}
# (codebook id, half-bits) pairs compiled (the reference's experts_grouped.cuh ESP_CASES)
COMPILED = {(1, k2) for k2 in range(2, 17, 2)} | {(3, 2), (3, 4), (3, 6), (6, 4), (6, 6), (6, 8), (7, 6), (7, 8),
                                                   (7, 10)}


def dequant(trellis: torch.Tensor, K: int, grid: int) -> torch.Tensor:
    """W [in, out] fp16 through the library's decode (bit-identical to the reference's)."""
    out = torch.empty((trellis.shape[0] * 16, trellis.shape[1] * 16), dtype=torch.float16, device=trellis.device)
    ext().dequant(trellis.contiguous(), out, 2 * K, KERNEL_CB[grid])
    return out
