"""Pin the CPU oracle against the REFERENCE plugin's own outputs (no GPU needed).

tests/golden/golden.npz holds outputs of the reference's CUDA extension (built from its sources by
oracle/build_ref.py, run on a B200 by tests/golden/make_golden.py) for the deterministic inputs of cases.py.

Bars: weight decode, full 65536-state codebook tables and the Hadamard kernel bit-exact; dense / MoE layer outputs
within the output-rounding floor plus 2e-3 (the reference sums on tensor cores in its own order, the oracle in fp64);
routing: the oracle's exact-logit expert sets equal the reference kernel's except on near-ties of the reference's own
fp32 logits (its own gate, tests/gpu_route.py:96-113).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import cases as C
import oracle as O

GOLD = Path(__file__).resolve().parent / "golden" / "golden.npz"
pytestmark = pytest.mark.skipif(not GOLD.exists(), reason="golden.npz not generated yet")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def rel(y, ref):
    return float(np.abs(y.astype(np.float64) - ref).max() / np.abs(ref).max())


@pytest.mark.parametrize("cb,k2", C.COMPILED)
def test_dequant_pinned(gold, cb, k2):
    T = C.dequant_case(cb, k2)
    assert str(gold[f"dq_{cb}_{k2}_in"]) == C.checksum(T)
    assert np.array_equal(O.bits16(O.dequant(T, k2 // 2, cb)), gold[f"dq_{cb}_{k2}"])


@pytest.mark.parametrize("cb", sorted(C.TABLE_CASES))
def test_codebook_table_pinned(gold, cb):
    """every one of the 65536 states, decoded by the reference's kernel"""
    assert np.array_equal(O.codebook_table(cb), gold[f"table_{cb}"])


def test_index_forms_follow_tables(gold):
    for cb, idx in ((6, 22), (7, 23)):
        q = O.codebook_table(idx).view(np.float16).astype(np.float32)
        c = np.float32(3.94921875) / np.float32(15.0 if cb == 6 else 31.0)
        assert np.array_equal((q * c).astype(np.float32).astype(np.float16).view(np.uint16), gold[f"table_{cb}"])


def test_had_pinned(gold):
    x, pre, post = C.had_case()
    assert np.array_equal(O.bits16(O.had(x, pre, post)), gold["had_pre_post"])
    assert np.array_equal(O.bits16(O.had(x, pre)), gold["had_pre"])


CASES = [(n, K, Ns, cb, k2, M, xdt) for n, K, Ns, cb, k2, Ms, xdt in C.DENSE_CASES for M in Ms]


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}-M{c[5]}" for c in CASES])
def test_dense_pinned(gold, case):
    name, K, Ns, cb, k2, M, xdt = case
    mats, xf = C.dense_inputs(name, K, Ns, cb, k2, M, xdt)
    assert str(gold[f"dense_{name}_{M}_in"]) == C.checksum(xf, *[m[0] for m in mats])
    want_bits = gold[f"dense_{name}_{M}"]
    want = C.bf16_to_f32(want_bits) if xdt == "bf16" else want_bits.view(np.float16).astype(np.float32)
    ref = np.concatenate([O.dense_matrix(xf, T, su, sv, k2 // 2, cb) for T, su, sv in mats], axis=1)
    floor = rel(ref.astype(np.float16 if xdt == "fp16" else np.float32) if xdt == "fp16" else
                C.bf16_to_f32(C.bf16_bits(ref)), ref)
    e = rel(want, ref)
    assert e < floor + 2e-3, f"reference kernel vs oracle: {e:.3e} (floor {floor:.3e})"


def test_route_pinned(gold):
    xb, gb, sb = C.route_inputs()
    pick, wts, lb = O.route(xb, gb, C.ROUTE_K, sb, C.ROUTE_E)
    rp, rw, rl = gold["route_pick"], gold["route_wts"], gold["route_logits"]
    k = C.ROUTE_K
    # the reference kernel's fp32 logits agree with the oracle's fp64 ones to fp32 accumulation error
    xf, gf = C.bf16_to_f32(xb).astype(np.float64), C.bf16_to_f32(gb).astype(np.float64)
    exact = xf @ gf.T
    assert np.abs(rl[:, :C.ROUTE_E] - exact).max() < 1e-4
    bad = 0
    for r in range(C.ROUTE_R):
        mine, theirs = set(pick[r, :k].tolist()), set(rp[r, :k].tolist())
        if mine != theirs:
            a, b = sorted(mine - theirs), sorted(theirs - mine)
            ref_l = C.bf16_to_f32(C.bf16_bits(rl[r, :C.ROUTE_E]))
            gap = abs(float(ref_l[b].min()) - float(lb[r, a].max()))
            bad += gap > float(np.abs(ref_l).max()) * 2 ** -7
        else:
            order = {int(e): j for j, e in enumerate(rp[r, :k])}
            for j, e in enumerate(pick[r, :k]):
                assert abs(float(wts[r, j]) - float(rw[r, order[int(e)]])) < 2e-3
        assert rp[r, k] == C.ROUTE_E
        assert abs(float(wts[r, k]) - float(rw[r, k])) < 1e-5      # shared gate sigmoid
    assert bad == 0
    # grouping of the reference's own picks equals the oracle's grouping rule
    uids, members, n = O.group(rp, C.ROUTE_E + 1)
    assert np.array_equal(uids, gold["route_uids"]) and np.array_equal(members, gold["route_members"])


def test_moe_pinned(gold):
    experts, xb, pick, wts, gate_w = C.moe_inputs()
    x = C.bf16_to_f32(xb)
    E = len(experts)
    # group_shared's tables: routed picks, then the shared slot with sigmoid(x . gate_w)
    pk = np.concatenate([pick, np.full((pick.shape[0], 1), E - 1, np.int32)], 1)
    sg = C.bf16_to_f32(gate_w).astype(np.float64)
    shared_w = (1 / (1 + np.exp(-(x.astype(np.float64) @ sg)))).astype(np.float32)
    wt = np.concatenate([wts, shared_w[:, None]], 1)
    assert np.array_equal(pk, gold["moe_pick"])
    assert np.abs(wt - gold["moe_wts"]).max() < 1e-6
    routed, shared, y = O.moe(x, pk, gold["moe_wts"], experts, C.MOE_K)
    ref_y = gold["moe_y"]
    assert rel(ref_y, y) < 2e-3
    out, osh = C.bf16_to_f32(gold["moe_out"]), C.bf16_to_f32(gold["moe_shared"])
    for got, want in ((out, routed), (osh, shared)):
        floor = rel(C.bf16_to_f32(C.bf16_bits(want)), want)
        assert rel(got, want) < floor + 2e-3
