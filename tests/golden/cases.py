"""Deterministic inputs of the golden cases, shared by make_golden.py (which runs the reference plugin's own CUDA
extension on a GPU to produce the outputs) and the tests (which regenerate the same inputs and compare).

Inputs are drawn with numpy's PCG64 from fixed seeds, so only outputs and a checksum of the inputs are stored in
golden.npz. Shapes and distributions follow the reference's own tests: random int16 trellises
(tests/gpu_grouped.py:145-147), +-1 suh, U(0.5, 1.5)/64-scaled +-1 svh, N(0, 1) activations, router rows with 1% of the
channels scaled by 4 (tests/gpu_route.py:79).
"""
from __future__ import annotations

import hashlib

import numpy as np

# (kernel codebook, half-bits) pairs of the reference (experts_grouped.cuh:227-229)
COMPILED = sorted({(1, k2) for k2 in range(2, 17, 2)} | {(3, 2), (3, 4), (3, 6), (6, 4), (6, 6), (6, 8), (7, 6),
                                                          (7, 8), (7, 10)})
TABLE_CASES = {1: 16, 3: 6, 6: 8, 7: 8}          # codebook -> k2 used to enumerate its full state table


def rng(*key) -> np.random.Generator:
    h = hashlib.sha256(repr(key).encode()).digest()
    return np.random.default_rng(int.from_bytes(h[:8], "little"))


def checksum(*arrays) -> str:
    m = hashlib.sha256()
    for a in arrays:
        m.update(np.ascontiguousarray(a).tobytes())
    return m.hexdigest()[:16]


def bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b).astype(np.uint32) << 16).view(np.float32)


def trellis(key, kin: int, n: int, K: int) -> np.ndarray:
    return rng("trellis", key).integers(-32768, 32768, size=(kin // 16, n // 16, 16 * K), dtype=np.int16)


def suh(key, k: int) -> np.ndarray:
    return np.where(rng("suh", key).random(k) < 0.5, -1.0, 1.0).astype(np.float16)


def svh(key, n: int) -> np.ndarray:
    r = rng("svh", key)
    s = np.where(r.random(n) < 0.5, -1.0, 1.0)
    return (s * r.uniform(0.5, 1.5, n) / 64).astype(np.float16)


def activations(key, m: int, k: int) -> np.ndarray:
    """float32 N(0, 1) values already rounded to bf16 (returned as bf16 bits)."""
    return bf16_bits(rng("x", key).standard_normal((m, k)).astype(np.float32))


# ---- dequant: every compiled pair on a 64 x 128 matrix ----
def dequant_case(cb: int, k2: int):
    return trellis(("dq", cb, k2), 64, 128, k2 // 2)


# ---- full codebook tables: a large random trellis whose states cover all 65536 values ----
def table_trellis(cb: int, k2: int, attempt: int = 0):
    return trellis(("tab", cb, k2, attempt), 1024, 1024, k2 // 2)


# ---- had ----
def had_case():
    r = rng("had")
    x = r.standard_normal((5, 256)).astype(np.float16)
    return x, suh("had-pre", 256), svh("had-post", 256)


# ---- dense layer cases: (name, K, [N per shard], cb, k2, M, x dtype) ----
DENSE_CASES = [
    ("int6_single", 512, [256], 7, 8, (1, 8, 32), "bf16"),
    ("int5_qkv", 256, [256, 128, 128], 6, 8, (5,), "bf16"),
    ("e2m1_2bit", 256, [128], 3, 4, (3,), "fp16"),
    ("mcg_6bit", 256, [128], 1, 12, (3,), "fp16"),
    ("int5_3bit", 512, [128, 128], 6, 6, (17,), "bf16"),
]


def dense_inputs(name: str, K: int, Ns, cb: int, k2: int, M: int, xdt: str):
    mats = [(trellis(("dense", name, i), K, n, k2 // 2), suh(("dense", name, i), K), svh(("dense", name, i), n))
            for i, n in enumerate(Ns)]
    xb = activations(("dense", name, M), M, K)
    x = bf16_to_f32(xb)
    if xdt == "fp16":
        x = x.astype(np.float16).astype(np.float32)
    return mats, x


# ---- routing ----
ROUTE_R, ROUTE_H, ROUTE_E, ROUTE_K = 32, 2048, 256, 8


def route_inputs():
    r = rng("route")
    x = r.standard_normal((ROUTE_R, ROUTE_H)).astype(np.float32)
    x *= 1 + 3 * (r.random(ROUTE_H) < 0.01)
    gate = (r.standard_normal((ROUTE_E, ROUTE_H)) / np.sqrt(ROUTE_H)).astype(np.float32)
    sgate = (r.standard_normal(ROUTE_H) / np.sqrt(ROUTE_H)).astype(np.float32)
    return bf16_bits(x), bf16_bits(gate), bf16_bits(sgate)


# ---- a small MoE layer with mixed widths and a shared expert ----
MOE_E, MOE_D, MOE_I, MOE_R, MOE_K = 16, 256, 128, 4, 4
MOE_WIDTHS = [(3, 2), (3, 4), (6, 6)]             # (kernel cb, k2): 1-bit E2M1, 2-bit E2M1, 3-bit int5
MOE_SHARED = (7, 8)                               # 4-bit int6


def moe_inputs():
    r = rng("moe")
    experts = []
    for e in range(MOE_E + 1):
        cb, k2 = MOE_SHARED if e == MOE_E else MOE_WIDTHS[int(r.integers(0, len(MOE_WIDTHS)))]
        K = k2 // 2
        ex = {}
        for p, (kin, n) in (("gate", (MOE_D, MOE_I)), ("up", (MOE_D, MOE_I)), ("down", (MOE_I, MOE_D))):
            ex[p] = (trellis(("moe", e, p), kin, n, K), K, cb, suh(("moe", e, p), kin), svh(("moe", e, p), n))
        experts.append(ex)
    x = activations("moe-x", MOE_R, MOE_D)
    pick = np.stack([r.permutation(MOE_E)[:MOE_K] for _ in range(MOE_R)]).astype(np.int32)
    w = np.exp(r.standard_normal((MOE_R, MOE_K)))
    wts = (w / w.sum(1, keepdims=True)).astype(np.float32)
    gate_w = bf16_bits((r.standard_normal(MOE_D) / np.sqrt(MOE_D)).astype(np.float32))
    return experts, x, pick, wts, gate_w
