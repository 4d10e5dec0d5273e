"""Trellis codebooks: how a checkpoint names them, which id the kernels use and which widths they decode.

A checkpoint marks a matrix's codebook with an `esp_grid` tensor (code 1 E2M1, 2 E4M3, 3 int5, 4 int6); without one,
a `mul1` marker means E2M1 and nothing means the stock mcg codebook (the reference's matrix.py:3-6, 33-37). The
library's kernels take codebook ids of their own numbering (1 mcg, 3 E2M1, 6 int5, 7 int6: the reference's
experts.py:34) and decode the (codebook, bits) pairs listed here (the reference's experts_grouped.cuh:227-229). E4M3
has no decode kernel, in the reference either.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Codebook:
    name: str
    grid: int                  # the checkpoint's code (0: stock mcg, no esp_grid tensor)
    kernel: int | None         # the library's codebook id; None: nothing decodes it
    widths: tuple[int, ...]    # bits a weight the kernels are compiled for


TABLE = (
    Codebook("mcg", 0, 1, (1, 2, 3, 4, 5, 6, 7, 8)),
    Codebook("e2m1", 1, 3, (1, 2, 3)),
    Codebook("e4m3", 2, None, ()),
    Codebook("int5", 3, 6, (2, 3, 4)),
    Codebook("int6", 4, 7, (3, 4, 5)),
)
BY_GRID = {c.grid: c for c in TABLE}
# grid code -> kernel id, for the codebooks that have a kernel (the reference's experts.KERNEL_CB)
KERNEL_CB = {c.grid: c.kernel for c in TABLE if c.kernel is not None}
# (kernel id, half-bits) pairs with a decode instance (the reference's experts.COMPILED)
COMPILED = frozenset((c.kernel, 2 * b) for c in TABLE if c.kernel is not None for b in c.widths)


def grid_code(tensors: dict) -> int:
    """The codebook code of one matrix's checkpoint tensors."""
    if "esp_grid" in tensors:
        code = int(tensors["esp_grid"].reshape(-1)[0].item())
        if code not in BY_GRID or code == 0:
            raise ValueError(f"esp_grid code {code} is not a known codebook (1 E2M1, 2 E4M3, 3 int5, 4 int6)")
        return code
    return 1 if "mul1" in tensors else 0


def kernel_id(grid: int, bits: int, what: str = "matrix") -> int:
    """The kernels' codebook id for a matrix of `bits` bits a weight; NotImplementedError when nothing decodes it."""
    book = BY_GRID.get(grid)
    if book is None or book.kernel is None:
        raise NotImplementedError(f"{what}: grid code {grid} has no decode kernel")
    if bits not in book.widths:
        raise NotImplementedError(f"{what}: no {book.name} decode at {bits} bits (built: {book.widths})")
    return book.kernel
