"""The two torch operators a vLLM model calls, so torch.compile and CUDA-graph capture see opaque calls.

Names, schemas and results are the reference plugin's (vllm_espalier/ops.py:54-87):

  espalier::matmul(Tensor x, Tensor trellis, Tensor suh, Tensor svh, int K, int cb) -> Tensor
      one coded matrix, x fp16 [m, in] -> fp16 [m, out] = H(H(x * suh) @ W) * svh
  espalier::dense(Tensor x, Tensor[] trellis, Tensor[] suh, Tensor[] svh, int key) -> Tensor
      every matrix of one registered layer (dense.Dense under `key`), x [m, in] -> [m, n_out] in x's dtype

Rows: up to 32 a kernel call. Above that (prefill) ESPALIER_PREFILL_MODE=chunk (default) runs 32-row windows, so a row
gets the same bits as in decode; =gemm decodes each matrix to fp16 once and multiplies with cuBLAS between the two
Hadamard passes (never for a layer of 2^28 weights or more: the LM head stays in windows).
"""
from __future__ import annotations

import itertools
import weakref

import torch

from ._env import PREFILL
from .dense import MAX_ROWS, Dense

if PREFILL not in ("chunk", "gemm"):
    raise ValueError(f"ESPALIER_PREFILL_MODE={PREFILL!r}: expected chunk or gemm")
GEMM_LIMIT = 1 << 28          # weights (in x out) from which a layer is never decoded to fp16 whole


class Registry:
    """dense.Dense objects by the integer key a compiled graph passes to espalier::dense."""

    def __init__(self):
        self._layers: dict[int, Dense] = {}
        self._keys = itertools.count()

    def add(self, d: Dense, owner=None) -> int:
        """Register d; with `owner`, the entry goes when the owner is garbage collected (a layer vLLM drops)."""
        key = next(self._keys)
        self._layers[key] = d
        if owner is not None:
            weakref.finalize(owner, self._layers.pop, key, None)
        return key

    def __getitem__(self, key: int) -> Dense:
        try:
            return self._layers[key]
        except KeyError:
            raise KeyError(f"espalier::dense: no layer registered under key {key}") from None

    def __contains__(self, key: int) -> bool:
        return key in self._layers


LAYERS = Registry()


def register_dense(d: Dense, owner=None) -> int:
    """Register a layer and return the key espalier::dense takes."""
    return LAYERS.add(d, owner)


def windowed(run, x: torch.Tensor, n_out: int, dtype) -> torch.Tensor:
    """run(rows, out) on consecutive MAX_ROWS-row windows of x, into one [m, n_out] output."""
    if x.shape[0] <= MAX_ROWS:
        return run(x, None)
    y = torch.empty((x.shape[0], n_out), dtype=dtype, device=x.device)
    for lo in range(0, x.shape[0], MAX_ROWS):
        run(x[lo:lo + MAX_ROWS], y[lo:lo + MAX_ROWS])
    return y


class _Single:
    """A one-matrix Dense per trellis, made on first use (the matmul op carries the tensors, not a layer)."""

    def __init__(self):
        self._cache: dict[tuple, Dense] = {}

    def get(self, trellis, suh, svh, K: int, cb: int) -> Dense:
        key = (trellis.data_ptr(), suh.data_ptr(), svh.data_ptr(), K, cb)
        d = self._cache.get(key)
        if d is None:
            class _M:   # the attributes Dense reads
                pass
            m = _M()
            m.trellis, m.suh, m.svh, m.K, m.cb = trellis, suh, svh, K, cb
            m.in_features, m.out_features = suh.numel(), svh.numel()
            d = self._cache[key] = Dense([m])
        return d


_SINGLES = _Single()


def decoded_gemm(x: torch.Tensor, trellis, suh, svh, K: int, cb: int) -> torch.Tensor:
    """The gemm prefill form of one matrix (the reference's ops.py:45-51): W decoded to fp16, H(x * suh) by the had
    kernel, the product by cuBLAS in fp16, then H(.) * svh by the had kernel."""
    from ._lib import ext
    from .matrix import dequant
    e = ext()
    xh = torch.empty_like(x)
    e.had(x, suh, None, xh)
    y = xh @ dequant(trellis, K, cb)
    e.had(y, None, svh, y)
    return y


def _matmul_impl(x, trellis, suh, svh, K, cb):
    if x.shape[0] > MAX_ROWS and PREFILL == "gemm":
        return decoded_gemm(x, trellis, suh, svh, K, cb)
    d = _SINGLES.get(trellis, suh, svh, K, cb)
    return windowed(lambda rows, out: d.forward(rows, out=out), x, d.n_out, x.dtype)


def _dense_impl(x, trellis, suh, svh, key):
    d = LAYERS[key]
    x = x.contiguous()
    if x.shape[0] > MAX_ROWS and PREFILL == "gemm" and d.K * d.N < GEMM_LIMIT:
        xh = x.to(torch.float16).contiguous()
        parts = [decoded_gemm(xh, t, s, v, m.K, m.cb) for t, s, v, m in zip(trellis, suh, svh, d.mats)]
        y = torch.cat(parts, dim=-1).to(x.dtype)
        return torch.nn.functional.pad(y, (0, d.n_out - d.N)) if d.n_out > d.N else y
    return windowed(lambda rows, out: d.forward(rows, trellis, suh, svh, out=out), x, d.n_out, x.dtype)


torch.library.define("espalier::matmul", "(Tensor x, Tensor trellis, Tensor suh, Tensor svh, int K, int cb) -> Tensor")
torch.library.define("espalier::dense", "(Tensor x, Tensor[] trellis, Tensor[] suh, Tensor[] svh, int key) -> Tensor")
torch.library.impl("espalier::matmul", "CUDA")(_matmul_impl)
torch.library.impl("espalier::dense", "CUDA")(_dense_impl)


@torch.library.register_fake("espalier::matmul")
def _matmul_shape(x, trellis, suh, svh, K, cb):
    return x.new_empty((x.shape[0], svh.shape[0]), dtype=torch.float16)


@torch.library.register_fake("espalier::dense")
def _dense_shape(x, trellis, suh, svh, key):
    return x.new_empty((x.shape[0], LAYERS[key].n_out))


def matmul(x, trellis, suh, svh, K: int, cb: int) -> torch.Tensor:
    return torch.ops.espalier.matmul(x, trellis, suh, svh, K, cb)


def dense(x, trellis, suh, svh, key: int) -> torch.Tensor:
    return torch.ops.espalier.dense(x, trellis, suh, svh, key)


__all__ = ["matmul", "dense", "register_dense", "LAYERS", "windowed", "decoded_gemm"]
