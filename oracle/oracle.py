"""numpy front end of the CPU oracle (liboracle.so, built from espalier_oracle.c by oracle/Makefile).

TEST INFRASTRUCTURE ONLY. tests/, the smoke check and bench.py's CPU-baseline leg use this module as the checker; the
product path never imports it. Each function names the reference code it restates (paths inside the reference plugin,
geodesa-ai/vllm-espalier).

Arrays of fp16 / bf16 values are passed as their uint16 bit patterns; helpers convert from numpy float16 and from
bf16 bits.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
HAD_SCALE = np.float32(0.08838834764831845)

# Espalier grid code (checkpoint esp_grid / EspMatrix.cb) -> kernel codebook id (vllm_espalier/experts.py:34)
KERNEL_CB = {0: 1, 1: 3, 3: 6, 4: 7}
# (kernel codebook, half-bits k2) pairs the reference compiles (experts_grouped.cuh:227-229)
COMPILED = sorted({(1, k2) for k2 in range(2, 17, 2)} | {(3, 2), (3, 4), (3, 6), (6, 4), (6, 6), (6, 8), (7, 6),
                                                          (7, 8), (7, 10)})


def _load():
    if not LIB.exists() or LIB.stat().st_mtime < (HERE / "espalier_oracle.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    lib = C.CDLL(str(LIB))
    P = C.c_void_p
    i, f, d = C.c_int, C.c_float, C.c_double
    sig = {
        "orc_h2f": (f, [C.c_uint16]), "orc_f2h": (C.c_uint16, [f]), "orc_d2h": (C.c_uint16, [d]),
        "orc_d2bf": (C.c_uint16, [d]), "orc_f2bf": (C.c_uint16, [f]), "orc_bf2f": (f, [C.c_uint16]),
        "orc_mcg": (C.c_uint16, [C.c_uint32]), "orc_codebook": (C.c_uint16, [i, C.c_uint32]),
        "orc_codebook_table": (None, [i, P]), "orc_int_step": (f, [i]),
        "orc_state": (C.c_uint32, [P, i, i]), "orc_states": (None, [P, i, i, i, P]),
        "orc_dequant": (i, [P, i, i, i, i, P]), "orc_dequant_f32": (i, [P, i, i, i, i, P]),
        "orc_fwht128": (None, [P]),
        "orc_rotate": (None, [P, i, i, P, P]), "orc_dense": (None, [P, P, i, i, i, P, f, P]),
        "orc_had": (None, [P, i, i, P, P, P]), "orc_router_logit": (d, [P, P, i]),
        "orc_group": (i, [P, i, i, i, P, P, i, i]),
        "orc_route": (None, [P, i, i, P, i, P, i, i, P, P, P]),
        "orc_gateup_epilogue": (None, [P, P, i, P, P, P, P]), "orc_down_epilogue": (None, [P, i, P, P]),
        "orc_combine_row": (None, [P, P, i, i, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    return lib


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


def bits16(a) -> np.ndarray:
    """uint16 bit patterns of a float16 array (or a uint16 / int16 array of bits)."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        return a.view(np.uint16)
    return a.astype(np.uint16, copy=False) if a.dtype != np.int16 else a.view(np.uint16)


def f16(bits: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(bits).view(np.float16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(bits).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """round-to-nearest-even float32 -> bf16 bits (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


# ---------------------------------------------------------------------------------------------------------------
# codebooks and geometry (experts_grouped.cuh:23-154, 330-339)
# ---------------------------------------------------------------------------------------------------------------

def codebook_table(cb: int) -> np.ndarray:
    """uint16 [65536]: fp16 bits of codebook cb (1 mcg, 3 E2M1, 6 int5, 7 int6, 22 / 23 int5 / int6 index)."""
    out = np.empty(65536, np.uint16)
    lib().orc_codebook_table(cb, _p(out))
    return out


def states(T: np.ndarray, K: int) -> np.ndarray:
    """trellis int16 [Kin/16, N/16, 16K] -> uint16 [Kin, N] trellis state of every weight."""
    T = np.ascontiguousarray(T, dtype=np.int16)
    KT, NT, L = T.shape
    assert L == 16 * K
    S = np.empty((KT * 16, NT * 16), np.uint16)
    lib().orc_states(_p(T), KT * 16, NT * 16, K, _p(S))
    return S


def dequant(T: np.ndarray, K: int, cb: int) -> np.ndarray:
    """W float16 [Kin, N] (experts_grouped.cuh:321-340 / experts.dequant), cb = kernel codebook id."""
    T = np.ascontiguousarray(T, dtype=np.int16)
    KT, NT, L = T.shape
    assert L == 16 * K, (T.shape, K)
    W = np.empty((KT * 16, NT * 16), np.uint16)
    rc = lib().orc_dequant(_p(T), KT * 16, NT * 16, K, cb, _p(W))
    if rc:
        raise ValueError(f"orc_dequant: error {rc}")
    return W.view(np.float16)


def dequant_f32(T: np.ndarray, K: int, cb: int) -> np.ndarray:
    """dequant's values widened to float32 [Kin, N], through the word-window decode (the timed CPU baseline's)."""
    T = np.ascontiguousarray(T, dtype=np.int16)
    KT, NT, L = T.shape
    assert L == 16 * K, (T.shape, K)
    W = np.empty((KT * 16, NT * 16), np.float32)
    rc = lib().orc_dequant_f32(_p(T), KT * 16, NT * 16, K, cb, _p(W))
    if rc:
        raise ValueError(f"orc_dequant_f32: error {rc}")
    return W


def int_step(cb: int) -> float:
    return float(lib().orc_int_step(cb))


def kernel_scale(cb: int) -> np.float32:
    """Grid step applied after accumulation when the kernels decode int5 / int6 as integer indices."""
    return np.float32(int_step(cb)) if cb in (6, 7) else np.float32(1.0)


# ---------------------------------------------------------------------------------------------------------------
# rotations and the dense layer (dense.cu)
# ---------------------------------------------------------------------------------------------------------------

def fwht128(v: np.ndarray) -> np.ndarray:
    v = np.ascontiguousarray(v, dtype=np.float32).copy()
    assert v.size == 128
    lib().orc_fwht128(_p(v))
    return v


def rotate(x: np.ndarray, suh: np.ndarray) -> np.ndarray:
    """xh float16 [M, K] = fp16(H(x * suh) / sqrt(128)) per 128-block (dense.cu:92-108); x float32 (exact values of
    the model's bf16 / fp16 input)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    suh = bits16(suh)
    xh = np.empty((M, K), np.uint16)
    lib().orc_rotate(_p(x), M, K, _p(suh), _p(xh))
    return xh.view(np.float16)


def dense_from_w(xh: np.ndarray, W: np.ndarray, svh: np.ndarray, scale=1.0) -> np.ndarray:
    """fp32 [M, N] finished outputs: per 128 columns H(xh @ W) * scale * (HAD * svh) (dense.cu:120-128); the dot
    products are accumulated in fp64."""
    xh, W, svh = bits16(xh), bits16(W), bits16(svh)
    M, K = xh.shape
    N = W.shape[1]
    y = np.empty((M, N), np.float32)
    lib().orc_dense(_p(xh), _p(W), M, K, N, _p(svh), float(scale), _p(y))
    return y


def dense_matrix(x: np.ndarray, T: np.ndarray, suh, svh, K: int, cb: int) -> np.ndarray:
    """One Espalier matrix, fp32 [M, N]: the reference decode-then-matmul composition
    y = H(H(x * suh) @ W) * svh with W the exact decoded weights and fp16 rotated activations."""
    W = dequant(T, K, cb)
    xh = rotate(x, suh)
    return dense_from_w(xh, W, svh, 1.0)


def had(x: np.ndarray, pre=None, post=None) -> np.ndarray:
    """fp16 H(x * pre) / sqrt(128) * post along rows of 128 (dense.cu:242-265)."""
    x = bits16(np.ascontiguousarray(x, dtype=np.float16))
    M, K = x.shape
    y = np.empty_like(x)
    lib().orc_had(_p(x), M, K, _p(None if pre is None else bits16(pre)), _p(None if post is None else bits16(post)),
                  _p(y))
    return y.view(np.float16)


# ---------------------------------------------------------------------------------------------------------------
# routing and grouping (route.cu, experts.cu:23-76)
# ---------------------------------------------------------------------------------------------------------------

def router_logit(x_bf16: np.ndarray, w_bf16: np.ndarray) -> float:
    x, w = bits16(x_bf16), bits16(w_bf16)
    return float(lib().orc_router_logit(_p(x), _p(w), x.size))


def route(x_bf16: np.ndarray, gate_bf16: np.ndarray, k: int, sgate_bf16=None, shared_id: int = -1):
    """x bf16 bits [R, H], gate bf16 bits [E, H] -> (pick int32 [R, k(+1)], wts float32, logits_bf16 as float32 [R, E])."""
    x, gate = bits16(x_bf16), bits16(gate_bf16)
    R, H = x.shape
    E = gate.shape[0]
    has = sgate_bf16 is not None and shared_id >= 0
    slots = k + has
    lb = np.empty((R, E), np.float32)
    pick = np.empty((R, slots), np.int32)
    wts = np.empty((R, slots), np.float32)
    lib().orc_route(_p(x), R, H, _p(gate), E, _p(bits16(sgate_bf16) if has else None), k, shared_id if has else -1,
                    _p(lb), _p(pick), _p(wts))
    return pick, wts, lb


def group(pick: np.ndarray, E: int, maxm: int | None = None, maxu: int | None = None):
    """(uids int32 [count], members int32 [count, maxm], count) in the reference's order."""
    pick = np.ascontiguousarray(pick, dtype=np.int32)
    R, slots = pick.shape
    maxm = R if maxm is None else maxm
    maxu = min(R * slots, E) if maxu is None else maxu
    uids = np.full(maxu, -1, np.int32)
    members = np.full((maxu, maxm), -1, np.int32)
    n = lib().orc_group(_p(pick), R, slots, E, _p(uids), _p(members), maxm, maxu)
    if n < 0:
        raise ValueError("grouping overflow")
    return uids[:n], members[:n], n


# ---------------------------------------------------------------------------------------------------------------
# MoE (experts.cu:97-393, experts.py routed2)
# ---------------------------------------------------------------------------------------------------------------

def gateup_epilogue(g: np.ndarray, u: np.ndarray, svh_g, svh_u, suh_d) -> np.ndarray:
    g = np.ascontiguousarray(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    xd = np.empty(g.size, np.uint16)
    lib().orc_gateup_epilogue(_p(g), _p(u), g.size, _p(bits16(svh_g)), _p(bits16(svh_u)), _p(bits16(suh_d)), _p(xd))
    return xd.view(np.float16)


def down_epilogue(z: np.ndarray, svh_d) -> np.ndarray:
    z = np.ascontiguousarray(z, np.float32)
    y = np.empty(z.size, np.float32)
    lib().orc_down_epilogue(_p(z), z.size, _p(bits16(svh_d)), _p(y))
    return y


def combine_row(y: np.ndarray, w: np.ndarray, n_routed: int) -> np.ndarray:
    y = np.ascontiguousarray(y, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty(y.shape[1], np.float32)
    lib().orc_combine_row(_p(y), _p(w), n_routed, y.shape[1], _p(out))
    return out


def _lin_sum(xh: np.ndarray, W: np.ndarray) -> np.ndarray:
    return (xh.astype(np.float64) @ W.astype(np.float64)).astype(np.float32)


def moe(x: np.ndarray, pick: np.ndarray, wts: np.ndarray, experts, n_routed: int):
    """One MoE layer for rows x (float32 exact values [R, D]) with slots pick / wts [R, slots] (the shared expert, if
    any, as the last slot), experts[e] = dict(gate=(T, K, cb, suh, svh), up=..., down=...) with kernel codebook ids.
    Returns (routed float32 [R, D], shared float32 [R, D] or None, y per slot float32 [R, slots, D]) before the
    model-dtype rounding (the caller rounds). Follows experts.py routed2 -> experts.cu kernels."""
    R, slots = pick.shape
    D = x.shape[1]
    cache = {}

    def W(e, which):
        key = (e, which)
        if key not in cache:
            T, K, cb = experts[e][which][:3]
            cache[key] = dequant_f32(T, K, cb)      # the same values as dequant's, through the faster decode
        return cache[key]

    y = np.zeros((R, slots, D), np.float32)
    for r in range(R):
        for q in range(slots):
            e = int(pick[r, q])
            if e < 0 or e >= len(experts):
                continue
            g, u, d = experts[e]["gate"], experts[e]["up"], experts[e]["down"]
            xg = rotate(x[r:r + 1], g[3])
            xu = rotate(x[r:r + 1], u[3])
            gs = _lin_sum(xg.astype(np.float32), W(e, "gate"))[0]
            us = _lin_sum(xu.astype(np.float32), W(e, "up"))[0]
            xd = gateup_epilogue(gs, us, g[4], u[4], d[3])
            ds = _lin_sum(xd.astype(np.float32)[None], W(e, "down"))[0]
            y[r, q] = down_epilogue(ds, d[4])
    routed = np.stack([combine_row(y[r, :n_routed], wts[r, :n_routed], n_routed) for r in range(R)])
    shared = None
    if slots > n_routed:
        shared = (wts[:, n_routed:n_routed + 1] * y[:, n_routed]).astype(np.float32)
    return routed, shared, y


def num_threads() -> int:
    return int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
