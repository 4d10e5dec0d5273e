"""CPU tests of the oracle and of the arithmetic choices the kernels make (no GPU).

* The oracle's IEEE helpers against numpy / torch conversions.
* The trellis geometry of the oracle against an independent bit-by-bit restatement of the reference's LaneMap /
  decode_tile window arithmetic (experts_grouped.cuh:83-154), including its 4-bit special path.
* The kernels' cheaper codebook formulations, checked exhaustively over all 65536 states against the reference's
  rules as restated by the oracle: E2M1 through a nudged fp32 scale and round-to-nearest-even e2m1 conversion, and the
  int5 / int6 index q through an fp32 magic-number add.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import cases as C
import oracle as O


def test_fp16_bf16_helpers():
    r = np.random.default_rng(0)
    xs = np.concatenate([r.standard_normal(4000).astype(np.float32) * s for s in (1e-6, 1e-3, 1, 300, 6e4)])
    lib = O.lib()
    assert all(lib.orc_f2h(float(v)) == int(np.float16(v).view(np.uint16)) for v in xs if abs(v) < 65504)
    allh = np.arange(0, 65536, 97, dtype=np.uint16)
    fin = np.isfinite(allh.view(np.float16))
    got = np.array([lib.orc_h2f(int(h)) for h in allh[fin]], np.float32)
    assert np.array_equal(got, allh[fin].view(np.float16).astype(np.float32))
    tb = torch.from_numpy(xs).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(O.f32_to_bf16(xs), tb)
    assert all(lib.orc_f2bf(float(v)) == int(b) for v, b in zip(xs[::37], tb[::37]))


def _state_reference_style(words: np.ndarray, K: int, p: int) -> int:
    """The reference's window arithmetic for one value: Fmt<K2>::end, LaneMap's (hi word, lo word, shift) and the
    64-bit merge (experts_grouped.cuh:83-109, 139-149), GV = 1 (one window a merge)."""
    K2, TW = 2 * K, 8 * K

    def end(q):
        return (q >> 1) * K2 + (K2 if q & 1 else K2 >> 1)
    last_end = end(p) + 128 * K2
    hr = (last_end - 1) >> 5
    hi, lo, sh = hr % TW, (hr + TW - 1) % TW, (hr + 1) * 32 - last_end
    mm = ((int(words[lo]) << 32) | int(words[hi])) >> sh
    return mm & 0xFFFF


@pytest.mark.parametrize("K", range(1, 9))
def test_geometry_matches_reference_window_arithmetic(K):
    r = np.random.default_rng(K)
    lib = O.lib()
    for _ in range(3):
        words = r.integers(0, 2 ** 32, size=8 * K, dtype=np.uint64).astype(np.uint32)
        for p in range(256):
            want = _state_reference_style(words, K, p)
            got = lib.orc_state(words.ctypes.data, K, p)
            assert got == want, (K, p)


def test_geometry_4bit_special_path():
    """K2 == 8 path of decode_tile: lane L's states from words L-1 and L by a funnel shift (experts_grouped.cuh:127-138)."""
    r = np.random.default_rng(4)
    w = r.integers(0, 2 ** 32, size=32, dtype=np.uint64).astype(np.uint32)
    lib = O.lib()
    for lane in range(32):
        prev, cur = int(w[(lane + 31) & 31]), int(w[lane])
        s = (((prev << 32) | cur) >> 20) & 0xFFFFFFFF
        st = [(s >> 8) & 0xFFFF, (s >> 4) & 0xFFFF, s & 0xFFFF, cur >> 16, (cur >> 12) & 0xFFFF, (cur >> 8) & 0xFFFF,
              (cur >> 4) & 0xFFFF, cur & 0xFFFF]
        for j in range(8):
            assert lib.orc_state(w.ctypes.data, 4, 8 * lane + j) == st[j]


def test_value_positions_cover_tile_once():
    lib = O.lib()
    import ctypes
    seen = set()
    for p in range(256):
        r, c = ctypes.c_int(), ctypes.c_int()
        lib.orc_value_pos(p, ctypes.byref(r), ctypes.byref(c))
        seen.add((r.value, c.value))
    assert len(seen) == 256


def _e2m1_rne(u: np.ndarray) -> np.ndarray:
    """round-to-nearest-even onto the E2M1 grid {0, .5, 1, 1.5, 2, 3, 4, 6}, saturating (cvt.rn.satfinite.e2m1x2)."""
    grid = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6])
    a = np.minimum(np.abs(u), 6.0)
    idx = np.clip(np.searchsorted(grid, a), 1, 7)
    lo, hi = grid[idx - 1], grid[idx]
    pick_hi = (a - lo > hi - a) | ((a - lo == hi - a) & (idx % 2 == 0))
    out = np.where(pick_hi, hi, lo)
    out = np.where(a <= 0, 0.0, out)
    return np.copysign(out, u)


def test_e2m1_kernel_formulation_exhaustive():
    """e2m1_units2 (trellis.cuh): u = v * fl32(fl32(1/C) (1 - 2^-20)), RNE to E2M1, * C == the reference's rule."""
    mcg = O.codebook_table(1).view(np.float16).astype(np.float32)
    kappa = np.float32(np.float32(1 / 0.75) * np.float32(1 - 2 ** -20))
    assert kappa == np.float32(float.fromhex("0x1.55554p+0"))
    u = (mcg * kappa).astype(np.float32)
    got = (_e2m1_rne(u.astype(np.float64)) * 0.75).astype(np.float16)
    want = O.codebook_table(3).view(np.float16)
    assert np.array_equal(got.view(np.uint16), want.view(np.uint16))


@pytest.mark.parametrize("cb,six", [(22, False), (23, True)])
def test_int_index_magic_exhaustive(cb, six):
    """int_index2 (trellis.cuh): fl32(fl32(v k) + M), M = 1.5 2^23 + 0x6420; the low half-word as fp16 minus 1056
    equals rintf(fl32(v k)) for every state (up to the sign of zero)."""
    mcg = O.codebook_table(1).view(np.float16).astype(np.float32)
    k = np.float32(float.fromhex("0x1.f660bap+2") if six else float.fromhex("0x1.e62c10p+1"))
    p = (mcg * k).astype(np.float32)
    s = (p + np.float32(12608544.0)).astype(np.float32)
    low = (s.view(np.uint32) & 0xFFFF).astype(np.uint16).view(np.float16).astype(np.float32)
    q = (low - np.float32(1056.0)).astype(np.float16)
    want = O.codebook_table(cb).view(np.float16)
    # equal as numbers; the magic add cannot produce -0 where rintf gives -0 for v * k in (-0.5, 0), which changes no
    # product or sum of the GEMV (the dequant path, which must be bit-exact, uses rintf itself)
    assert np.array_equal(q.astype(np.float32), want.astype(np.float32))
    differ = q.view(np.uint16) != want.view(np.uint16)
    assert np.all(want[differ] == 0) and np.all(np.signbit(want[differ]))


def test_int6_single_fma_constant_exhaustive():
    """int_index2<7> (trellis.cuh) snaps with one FFMA, k' = INT6_K + 1 ulp: the exactly rounded v k' equals
    rintf(fl32(v k)) for every state (and no such constant exists for int5, which keeps FMUL + FADD)."""
    mcg = O.codebook_table(1).view(np.float16).astype(np.float64)
    k = np.float32(float.fromhex("0x1.f660bap+2"))
    kp = np.array([int(k.view(np.uint32)) + 1], np.uint32).view(np.float32)[0]
    assert float(kp) == float.fromhex("0x1.f660bcp+2")
    q = np.rint(mcg * float(kp))            # v * k' is exact in double; one round-half-even
    assert np.array_equal(q, O.codebook_table(23).view(np.float16).astype(np.float64))


@pytest.mark.parametrize("cb,idx,c_hi,c_lo", [(6, 22, 0x3436, 0x0666), (7, 23, 0x3014, 0x8319)])
def test_int_weight_two_term_exhaustive(cb, idx, c_hi, c_lo):
    """int_weight2 (trellis.cuh), the GEMVs' int5 / int6 weights: w = fl16(q c_hi + fl16(q c_lo)) from the index q
    (one fp16 multiply, one fp16 fused multiply-add) equals the reference's fl16(fl32(q c)) for every state, up to the
    sign of zero. The fp16 products are emulated exactly in float64 and rounded once."""
    q = O.codebook_table(idx).view(np.float16).astype(np.float64)
    hi, lo = (np.array([v], np.uint16).view(np.float16).astype(np.float64)[0] for v in (c_hi, c_lo))
    c = np.float32(3.94921875) / np.float32(15.0 if cb == 6 else 31.0)
    assert hi == np.float64(np.float16(c)) and lo == np.float64(np.float16(np.float64(c) - hi))
    r = (q * lo).astype(np.float16).astype(np.float64)        # HMUL2: the exact product rounded to fp16
    w = (q * hi + r).astype(np.float16)                        # HFMA2: exact q * c_hi + r, rounded once
    want = O.codebook_table(cb).view(np.float16)
    assert np.array_equal(w.astype(np.float32), want.astype(np.float32))


def test_int_grid_value_from_index():
    """c * q in fp32 rounded to fp16 (the exact form) for every state."""
    for cb, idx in ((6, 22), (7, 23)):
        q = O.codebook_table(idx).view(np.float16).astype(np.float32)
        c = np.float32(3.94921875) / np.float32(15.0 if cb == 6 else 31.0)
        got = (q * c).astype(np.float32).astype(np.float16)
        assert np.array_equal(got.view(np.uint16), O.codebook_table(cb))


def test_fwht_matches_sylvester():
    h = np.ones((1, 1))
    while h.shape[0] < 128:
        h = np.block([[h, h], [h, -h]])
    v = np.random.default_rng(1).standard_normal(128).astype(np.float32)
    np.testing.assert_allclose(O.fwht128(v), v.astype(np.float64) @ h, rtol=1e-5, atol=1e-4)


def test_grouping_order():
    pick = np.array([[3, 1, 7], [1, 5, 3]], np.int32)
    uids, members, n = O.group(pick, E=8)
    assert n == 4 and list(uids) == [1, 3, 5, 7]
    assert list(members[0]) == [0 * 32 + 1, 1 * 32 + 0] and list(members[1]) == [0 * 32 + 0, 1 * 32 + 2]
    assert list(members[2]) == [1 * 32 + 1, -1] and list(members[3]) == [0 * 32 + 2, -1]


def test_route_ties_lowest_id_and_order():
    xb, gb, sb = C.route_inputs()
    pick, wts, lb = O.route(xb[:4], gb, 8, sb, 256)
    for r in range(4):
        ids = pick[r, :8]
        vals = lb[r, ids]
        assert np.all(np.diff(vals) <= 0)
        rest = np.setdiff1d(np.arange(256), ids)
        assert lb[r, rest].max() <= vals.min()
        assert pick[r, 8] == 256
        assert abs(float(wts[r, :8].sum()) - 1) < 1e-6


@pytest.mark.parametrize("cb,k2", C.COMPILED)
def test_word_window_decode_matches_bit_serial(cb, k2):
    """The timed CPU baseline's decode (64-bit word windows, fp32 out) gives the oracle's weights bit for bit."""
    T = C.trellis(("f32-decode", cb, k2), 64, 256, k2 // 2)
    want = O.dequant(T, k2 // 2, cb).astype(np.float32)
    got = O.dequant_f32(T, k2 // 2, cb)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
