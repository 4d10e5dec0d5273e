"""ctypes binding of libespalier_b200.so and the reference-shaped extension object `ext()`.

`ext()` exposes the function names and argument orders of the reference's pybind module
(vllm_espalier/csrc/experts.cpp:234-248), taking torch tensors, checking them like the reference's TORCH_CHECKs and
raising RuntimeError with the library's message on any error status. Kernels are enqueued on torch's current CUDA
stream. ESPALIER_PREBUILT_EXTENSION may point at a prebuilt copy of the library (the reference's switch,
vllm_espalier/experts.py:44).
"""
from __future__ import annotations

import ctypes as C
import os
from functools import lru_cache
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIB_NAME = "libespalier_b200.so"

DTYPE = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}

ESP_OK, ESP_ERR_INVALID, ESP_ERR_UNSUPPORTED, ESP_ERR_SCRATCH, ESP_ERR_CUDA, ESP_ERR_TIMEOUT = range(6)


class EspError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


class esp_matrix_t(C.Structure):
    _fields_ = [("trellis", C.c_void_p), ("suh", C.c_void_p), ("svh", C.c_void_p), ("n", C.c_int),
                ("col0", C.c_int)]


P, I, L, S, F = C.c_void_p, C.c_int, C.c_longlong, C.c_size_t, C.c_float
SIGNATURES = {
    "esp_version": (I, []),
    "esp_last_error": (C.c_char_p, []),
    "esp_device_status": (I, [C.POINTER(C.c_int), I]),
    "esp_sm_count": (I, []),
    "esp_dequant": (I, [P, I, I, I, I, P, P]),
    "esp_had": (I, [P, I, I, P, P, P, P]),
    "esp_dense": (I, [P, I, L, I, I, C.POINTER(esp_matrix_t), I, I, I, P, I, L, P, S, P, S, P, I, P]),
    "esp_dense_noalloc": (I, [P, I, L, I, I, C.POINTER(esp_matrix_t), I, I, I, P, I, L, P]),
    "esp_dense_xh_bytes": (S, [I, I, I]),
    "esp_dense_z_bytes": (S, [I]),
}


def library_path() -> Path:
    p = os.environ.get("ESPALIER_PREBUILT_EXTENSION")
    return Path(p) if p else HERE / LIB_NAME


@lru_cache(1)
def lib():
    path = library_path()
    if not path.exists():
        raise RuntimeError(f"{path} is missing: build it with `make -C {HERE}` (or __graft_entry__.build())")
    h = C.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(h, name)
        fn.restype, fn.argtypes = res, args
    return h


def check(rc: int):
    if rc != ESP_OK:
        raise EspError(rc, lib().esp_last_error().decode() or f"espalier_b200 error {rc}")


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _need(cond: bool, msg: str):
    if not cond:
        raise RuntimeError(msg)


def _check(t: torch.Tensor, dtype: torch.dtype, name: str):
    _need(t.is_cuda and t.dtype == dtype and t.is_contiguous(), f"{name}: expected a contiguous CUDA tensor of the right dtype")


class _Ext:
    """The reference extension's functions over the C ABI."""

    # ---- dense layer (experts.cpp:193-211) ----
    @staticmethod
    def dense(x, T, suh, svh, col0, y, xh, Z, counters, k2, cb, SK=1, W=4, PF=1, rot_smem=0):
        """SK / W / PF / rot_smem are the reference's tile-plan hints; this library plans its own tiling (stream-K over
        all SMs) from the shape alone, so they are accepted and ignored."""
        _need(x.is_cuda and x.dim() == 2 and x.stride(1) == 1, "x: CUDA [M, K], unit column stride")
        _need(y.is_cuda and y.dim() == 2 and y.stride(1) == 1, "y: CUDA [M, N], unit column stride")
        _need(len(T) == len(suh) == len(svh) == len(col0), "one entry a matrix")
        _need(x.dtype in DTYPE and y.dtype in DTYPE, "x / y dtype must be fp16, bf16 or fp32")
        M, K = x.shape
        mats = (esp_matrix_t * len(T))()
        for i, (t, su, sv, c0) in enumerate(zip(T, suh, svh, col0)):
            _need(t.is_cuda and t.dtype == torch.int16 and t.is_contiguous() and t.dim() == 3,
                  "trellis: contiguous int16 [K/16, N/16, 16K]")
            _check(su, torch.float16, "suh")
            _check(sv, torch.float16, "svh")
            _need(int(c0) + sv.numel() <= y.size(1), "matrix columns past y")
            _need(t.size(0) * 16 == K and t.size(1) * 16 == sv.numel() and t.size(2) == 8 * k2, "matrix shape")
            mats[i] = esp_matrix_t(t.data_ptr(), su.data_ptr(), sv.data_ptr(), sv.numel(), int(c0))
        _check(Z, torch.float32, "Z")
        _check(counters, torch.int32, "counters")
        _need(xh.is_cuda and xh.is_contiguous(), "xh: contiguous CUDA scratch")
        check(lib().esp_dense(x.data_ptr(), DTYPE[x.dtype], x.stride(0), M, K, mats, len(T), int(k2), int(cb),
                              y.data_ptr(), DTYPE[y.dtype], y.stride(0), xh.data_ptr(), xh.numel() * xh.element_size(),
                              Z.data_ptr(), Z.numel() * 4, counters.data_ptr(), counters.numel(),
                              stream_ptr(x.device)))

    # ---- weight decode (experts.cpp:68-77) ----
    @staticmethod
    def dequant(T, out, k2, cb):
        _need(T.is_cuda and T.dtype == torch.int16 and T.is_contiguous() and T.dim() == 3,
              "T: int16 [K/16, N/16, 8 * k2]")
        _need(T.size(2) == 8 * k2, "trellis last dim must be 8 * k2")
        _check(out, torch.float16, "out")
        K, N = T.size(0) * 16, T.size(1) * 16
        _need(out.numel() == K * N, "out must be [K, N]")
        check(lib().esp_dequant(T.data_ptr(), K, N, int(k2), int(cb), out.data_ptr(), stream_ptr(T.device)))

    # ---- Hadamard transform (experts.cpp:226-232) ----
    @staticmethod
    def had(x, pre, post, y):
        _check(x, torch.float16, "x")
        _check(y, torch.float16, "y")
        M, K = x.shape
        check(lib().esp_had(x.data_ptr(), M, K, ptr(pre), ptr(post), y.data_ptr(), stream_ptr(x.device)))


@lru_cache(1)
def ext() -> _Ext:
    lib()
    return _Ext()


def device_status(reset: bool = True) -> int:
    v = C.c_int(0)
    check(lib().esp_device_status(C.byref(v), int(reset)))
    return v.value
