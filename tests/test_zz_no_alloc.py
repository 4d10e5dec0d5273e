"""The allocation-free dense entry point (esp_dense_noalloc) against the existing one (esp_dense), through the C ABI.

esp_dense_noalloc exists for callers that cannot allocate device memory when they run a layer: a serving engine whose
KV cache already holds nearly all of HBM, a host bound only through the C ABI with no allocator of its own, or a path
that must not take cudaMalloc's implicit synchronisation. Its scratch is one fixed array of device memory shared by
every call, so this test makes two calls in a row (the second reuses what the first left there) and checks both
against esp_dense with caller-provided scratch, and against the CPU oracle, with the dense tests' tolerances.

This file is collected last on purpose (a failure here leaves every other test already run).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

import cases as Cs
import oracle as O
from helpers import f32, floor_err, rel_err

from vllm_espalier_b200 import _lib

pytestmark = pytest.mark.gpu


def _layer(name, K, Ns, cb, k2, M, dev):
    mats, xf = Cs.dense_inputs(name, K, Ns, cb, k2, M, "bf16")
    keep = []
    arr = (_lib.esp_matrix_t * len(mats))()
    col = 0
    for i, (T, su, sv) in enumerate(mats):
        t, a, b = (torch.from_numpy(np.ascontiguousarray(v)).to(dev) for v in (T, su, sv))
        keep += [t, a, b]
        arr[i] = _lib.esp_matrix_t(t.data_ptr(), a.data_ptr(), b.data_ptr(), sv.size, col)
        col += sv.size
    ref = np.concatenate([O.dense_matrix(xf, T, su, sv, k2 // 2, cb) for T, su, sv in mats], axis=1)
    x = torch.from_numpy(xf).to(dev).to(torch.bfloat16)
    return arr, keep, x, col, ref


def _call_dense(lib, arr, n, x, N, k2, cb, dev):
    M, K = x.shape
    y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    xh = torch.empty(lib.esp_dense_xh_bytes(M, K, n) // 2, dtype=torch.float16, device=dev)
    z = torch.zeros(lib.esp_dense_z_bytes(M) // 4 + 1, dtype=torch.float32, device=dev)   # zero on entry
    cnt = torch.zeros(N // 128, dtype=torch.int32, device=dev)
    rc = lib.esp_dense(x.data_ptr(), 1, x.stride(0), M, K, arr, n, k2, cb, y.data_ptr(), 1, y.stride(0),
                       xh.data_ptr(), xh.numel() * 2, z.data_ptr(), z.numel() * 4, cnt.data_ptr(), cnt.numel(),
                       _lib.stream_ptr(dev))
    assert rc == 0, lib.esp_last_error()
    return y


def _call_noalloc(lib, arr, n, x, N, k2, cb, dev):
    M, K = x.shape
    y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    rc = lib.esp_dense_noalloc(x.data_ptr(), 1, x.stride(0), M, K, arr, n, k2, cb, y.data_ptr(), 1, y.stride(0),
                               _lib.stream_ptr(dev))
    assert rc == 0, lib.esp_last_error()
    return y


# (name, K, [N per matrix], cb, k2, M): a merged 3-matrix layer at 1 and 17 rows, then a different shape that reuses
# the shared scratch right after
CALLS = [("int5_qkv", 256, [256, 128, 128], 6, 8, 1), ("int5_qkv", 256, [256, 128, 128], 6, 8, 17),
         ("int6_single", 512, [256], 7, 8, 32)]


def test_noalloc_matches_dense_twice_in_a_row(dev):
    lib = _lib.lib()
    for name, K, Ns, cb, k2, M in CALLS:
        arr, keep, x, N, ref = _layer(name, K, Ns, cb, k2, M, dev)
        want = _call_dense(lib, arr, len(Ns), x, N, k2, cb, dev)
        first = _call_noalloc(lib, arr, len(Ns), x, N, k2, cb, dev)
        second = _call_noalloc(lib, arr, len(Ns), x, N, k2, cb, dev)
        torch.cuda.synchronize()
        for got in (first, second):
            # the same kernels, scratch layout and launch order as esp_dense: the same bits
            assert torch.equal(got, want), f"{name} M={M}: differs from esp_dense"
            e, fl = rel_err(f32(got), ref), floor_err(ref, torch.bfloat16)
            assert e < 1e-2 and e < fl + 2e-3, f"{name} M={M}: max rel err {e:.3e} (floor {fl:.3e})"
        assert torch.equal(first, second)
    assert _lib.device_status() == 0


def test_noalloc_allocates_no_device_memory(dev):
    """After one warm-up call (its first call on a device looks up the array's address), further calls leave the
    device's free memory unchanged: outputs are allocated before the measurement, the calls go straight to the C ABI."""
    lib = _lib.lib()
    name, K, Ns, cb, k2, M = CALLS[0]
    arr, keep, x, N, _ = _layer(name, K, Ns, cb, k2, M, dev)
    ys = [torch.empty((M, N), dtype=torch.bfloat16, device=dev) for _ in range(4)]
    stream = _lib.stream_ptr(dev)

    def call(y):
        rc = lib.esp_dense_noalloc(x.data_ptr(), 1, x.stride(0), M, K, arr, len(Ns), k2, cb, y.data_ptr(), 1,
                                   y.stride(0), stream)
        assert rc == 0, lib.esp_last_error()
    call(ys[0])
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(dev)
    for y in ys[1:]:
        call(y)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(dev)
    assert free1 == free0, f"free device memory moved by {free0 - free1} bytes"
    assert all(torch.equal(y, ys[0]) for y in ys[1:])


def test_noalloc_rejects_sizes_beyond_its_array(dev):
    lib = _lib.lib()
    arr = (_lib.esp_matrix_t * 1)(_lib.esp_matrix_t(16, 16, 16, 128, 0))
    rc = lib.esp_dense_noalloc(C.c_void_p(16), 1, 8192, 1, 8192, arr, 1, 8, 7, C.c_void_p(16), 1, 128, None)
    assert rc == _lib.ESP_ERR_INVALID and b"static scratch limit" in lib.esp_last_error()
