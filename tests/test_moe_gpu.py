"""GPU parity of the MoE path against the CPU oracle (and the reference's own outputs in golden.npz):
fused routing (ids bit-exact, weights within 2e-3, grouping exact, injected near-ties), group / group_shared, the
fused 4-launch pipeline (routed2) and the reference-kernel sequence (routed), row invariance and graph == eager
(the reference's tests/gpu_route.py, gpu_grouped.py, gpu_grouped_shared.py gates, on synthetic data)."""
from __future__ import annotations

import functools

import numpy as np
import pytest
import torch

import cases as C
import oracle as O
from helpers import f32, rel_err

from vllm_espalier_b200 import _lib
from vllm_espalier_b200 import experts as G

pytestmark = pytest.mark.gpu
GRID_OF = {1: 0, 3: 1, 6: 3, 7: 4}


class Mat:
    def __init__(self, T, K, cb, suh, svh, dev):
        self.trellis = torch.from_numpy(np.ascontiguousarray(T)).to(dev)
        self.suh = torch.from_numpy(suh).to(dev)
        self.svh = torch.from_numpy(svh).to(dev)
        self.K, self.cb = K, GRID_OF[cb]
        self.in_features, self.out_features = T.shape[0] * 16, T.shape[1] * 16


def bf(a_bits, dev):
    return torch.from_numpy(np.ascontiguousarray(a_bits).view(np.int16)).to(dev).view(torch.bfloat16)


def build(experts_np, dev):
    mats = [tuple(Mat(*ex[p], dev) for p in ("gate", "up", "down")) for ex in experts_np]
    return mats


# ---------------------------------------------------------------------------------------------------------------
# routing
# ---------------------------------------------------------------------------------------------------------------
def _route_tensors(R, E, k, dev, has=True):
    slots = k + has
    P = R * slots
    maxu = min(P, E + has)
    t = dict(logits=torch.zeros(R * (E + 1), dtype=torch.float32, device=dev),
             counter=torch.zeros(1, dtype=torch.int32, device=dev),
             pick=torch.zeros(P, dtype=torch.int32, device=dev), wts=torch.zeros(P, dtype=torch.float32, device=dev),
             uids=torch.zeros(maxu, dtype=torch.int32, device=dev), ucount=torch.zeros(1, dtype=torch.int32, device=dev),
             members=torch.full((maxu, R), -1, dtype=torch.int32, device=dev))
    return t


def _near_tie_rows(xb, gb, k, frac=0.05, seed=1):
    """Perturb 5% of the rows so that the fp64 logit gap between ranks k and k+1 is below 1e-3."""
    r = np.random.default_rng(seed)
    x = C.bf16_to_f32(xb).astype(np.float64)
    g = C.bf16_to_f32(gb).astype(np.float64)
    rows = r.choice(x.shape[0], max(1, int(frac * x.shape[0])), replace=False)
    for i in rows:
        lg = g @ x[i]
        order = np.argsort(-lg)
        a, b = order[k - 1], order[k]
        d = g[a] - g[b]
        gap = lg[a] - lg[b]
        xi = x[i] - d * (gap - r.uniform(-5e-4, 5e-4)) / (d @ d)
        x[i] = C.bf16_to_f32(C.bf16_bits(xi.astype(np.float32)))
    return C.bf16_bits(x.astype(np.float32)), rows


@pytest.mark.parametrize("R", [1, 7, 32])
def test_route_exact_ids(dev, R):
    xb, gb, sb = C.route_inputs()
    xb = xb[:R].copy()
    xb, tie_rows = _near_tie_rows(xb, gb, C.ROUTE_K)
    k, E = C.ROUTE_K, C.ROUTE_E
    t = _route_tensors(R, E, k, dev)
    _lib.ext().route_group(bf(xb, dev), bf(gb, dev), bf(sb, dev), k, E, t["logits"], t["counter"], t["pick"],
                           t["wts"], t["uids"], t["ucount"], t["members"])
    torch.cuda.synchronize()
    pick, wts, lb = O.route(xb, gb, k, sb, E)
    assert np.array_equal(t["pick"].cpu().numpy().reshape(R, k + 1), pick), "expert ids must match bit for bit"
    assert np.abs(t["wts"].cpu().numpy().reshape(R, k + 1)[:, :k] - wts[:, :k]).max() < 2e-3
    assert np.abs(t["wts"].cpu().numpy().reshape(R, k + 1)[:, k] - wts[:, k]).max() < 1e-5
    # exact routing: fp64 logits rounded once to bf16 (any order of summation), ties to the lowest id
    ex = C.bf16_to_f32(C.bf16_bits((C.bf16_to_f32(xb).astype(np.float64) @ C.bf16_to_f32(gb).astype(np.float64).T)
                                   .astype(np.float32)))
    for r in range(R):
        order = sorted(range(E), key=lambda e: (-ex[r, e], e))[:k]
        assert set(order) == set(pick[r, :k].tolist())
    uids, members, n = O.group(pick, E + 1)
    assert int(t["ucount"].item()) == n
    assert np.array_equal(t["uids"].cpu().numpy()[:n], uids)
    assert np.array_equal(t["members"].cpu().numpy()[:n], members)
    assert int(t["counter"].item()) == 0


def test_route_matches_reference_fixture(dev):
    """The reference kernel's (fp32-logit) choices equal ours except on its own near-ties (golden.npz)."""
    from pathlib import Path
    gold = Path(__file__).resolve().parent / "golden" / "golden.npz"
    if not gold.exists():
        pytest.skip("golden.npz missing")
    g = np.load(gold)
    xb, gb, sb = C.route_inputs()
    R, k, E = C.ROUTE_R, C.ROUTE_K, C.ROUTE_E
    t = _route_tensors(R, E, k, dev)
    _lib.ext().route_group(bf(xb, dev), bf(gb, dev), bf(sb, dev), k, E, t["logits"], t["counter"], t["pick"],
                           t["wts"], t["uids"], t["ucount"], t["members"])
    ours = t["pick"].cpu().numpy().reshape(R, k + 1)
    same = sum(set(ours[r, :k]) == set(g["route_pick"][r, :k]) for r in range(R))
    assert same >= R - 1


def test_group_and_group_shared(dev):
    R, k, E = 5, 4, 16
    r = np.random.default_rng(3)
    pick = np.stack([r.permutation(E)[:k] for _ in range(R)]).astype(np.int32)
    wts = r.random((R, k)).astype(np.float32)
    ids = torch.zeros(min(R * k, E), dtype=torch.int32, device=dev)
    cnt = torch.zeros(1, dtype=torch.int32, device=dev)
    mem = torch.full((ids.numel(), R), -1, dtype=torch.int32, device=dev)
    _lib.ext().group(torch.from_numpy(pick).to(dev), ids, cnt, mem, R, k, E)
    u, m, n = O.group(pick, E, maxu=ids.numel())
    assert int(cnt.item()) == n and np.array_equal(ids.cpu().numpy()[:n], u) and np.array_equal(mem.cpu().numpy()[:n], m)
    # group_shared: shared slot E with sigmoid(x . gate_w)
    xb = C.activations("gs-x", R, 256)
    gw = C.bf16_bits((r.standard_normal(256) / 16).astype(np.float32))
    P = R * (k + 1)
    po = torch.zeros(P, dtype=torch.int32, device=dev)
    wo = torch.zeros(P, dtype=torch.float32, device=dev)
    ids2 = torch.zeros(min(P, E + 1), dtype=torch.int32, device=dev)
    mem2 = torch.full((ids2.numel(), R), -1, dtype=torch.int32, device=dev)
    x = bf(xb, dev)
    _lib.ext().group_shared(torch.from_numpy(pick).to(dev), torch.from_numpy(wts).to(dev), x, x.stride(0), bf(gw, dev),
                            E, po, wo, ids2, cnt, mem2, R, k, E + 1)
    pk = np.concatenate([pick, np.full((R, 1), E, np.int32)], 1)
    assert np.array_equal(po.cpu().numpy().reshape(R, k + 1), pk)
    sw = 1 / (1 + np.exp(-(C.bf16_to_f32(xb).astype(np.float64) @ C.bf16_to_f32(gw).astype(np.float64))))
    assert np.abs(wo.cpu().numpy().reshape(R, k + 1)[:, k] - sw).max() < 1e-5
    u, m, n = O.group(pk, E + 1, maxu=ids2.numel())
    assert int(cnt.item()) == n and np.array_equal(mem2.cpu().numpy()[:n], m)


# ---------------------------------------------------------------------------------------------------------------
# the MoE layer
# ---------------------------------------------------------------------------------------------------------------
@pytest.fixture(scope="module")
def small_moe(dev):
    experts_np, xb, pick, wts, gate_w = C.moe_inputs()
    mats = build(experts_np, dev)
    L = G.prepare(mats[:-1], mats[-1], bf(gate_w, dev))
    return experts_np, xb, pick, wts, gate_w, L


def _oracle_moe(experts_np, xb, pick, wts, gate_w, k):
    x = C.bf16_to_f32(xb)
    E = len(experts_np)
    pk = np.concatenate([pick, np.full((pick.shape[0], 1), E - 1, np.int32)], 1)
    sw = (1 / (1 + np.exp(-(x.astype(np.float64) @ C.bf16_to_f32(gate_w).astype(np.float64))))).astype(np.float32)
    wt = np.concatenate([wts, sw[:, None]], 1)
    routed, shared, _ = O.moe(x, pk, wt, experts_np, k)
    return routed, shared


def test_routed2_vs_oracle_and_reference(dev, small_moe):
    experts_np, xb, pick, wts, gate_w, L = small_moe
    R, k = pick.shape
    s = G.scratch(L, 32, k + 1, dev)
    x = bf(xb, dev)
    out, sh = G.routed2(x, torch.from_numpy(pick).to(dev), torch.from_numpy(wts).to(dev), L, s)
    torch.cuda.synchronize()
    routed, shared = _oracle_moe(experts_np, xb, pick, wts, gate_w, k)
    for got, want in ((out, routed), (sh, shared)):
        e = rel_err(f32(got), want)
        fl = rel_err(C.bf16_to_f32(C.bf16_bits(want)), want)
        assert e < 1e-2 and e < fl + 2e-3, f"max rel err {e:.3e} (floor {fl:.3e})"
    from pathlib import Path
    gold = Path(__file__).resolve().parent / "golden" / "golden.npz"
    if gold.exists():
        g = np.load(gold)
        assert rel_err(f32(out), C.bf16_to_f32(g["moe_out"])) < 1e-2
        assert rel_err(f32(sh), C.bf16_to_f32(g["moe_shared"])) < 1e-2
    assert _lib.device_status() == 0
    assert int(s.cnt_gu.abs().sum()) == 0 and int(s.cnt_d.abs().sum()) == 0


def test_routed_reference_sequence(dev, small_moe):
    """The reference's separate kernels (group, rot_in, grouped Z, gateup_epilogue, grouped Z, down_combine)."""
    experts_np, xb, pick, wts, gate_w, L0 = small_moe
    mats = build(experts_np, dev)
    L = G.prepare(mats[:-1])                       # routed experts only, fp32 combine over all slots
    R, k = pick.shape
    s = G.scratch(L, 32, k, dev)
    x = bf(xb, dev)
    out = G.routed(x, torch.from_numpy(pick).to(dev), torch.from_numpy(wts).to(dev), L, s)
    torch.cuda.synchronize()
    routed, _, _ = O.moe(C.bf16_to_f32(xb), pick, wts, experts_np[:-1], k)
    assert rel_err(f32(out), routed) < 2e-3


def test_rows_alone_equal_window_and_graph(dev, small_moe):
    experts_np, xb, pick, wts, gate_w, L = small_moe
    R, k = pick.shape
    s = G.scratch(L, 32, k + 1, dev)
    x = bf(xb, dev)
    pk, wt = torch.from_numpy(pick).to(dev), torch.from_numpy(wts).to(dev)
    out, sh = G.routed2(x, pk, wt, L, s)
    out, sh = out.clone(), sh.clone()
    for r in range(R):
        o1, s1 = G.routed2(x[r:r + 1].contiguous(), pk[r:r + 1].contiguous(), wt[r:r + 1].contiguous(), L, s)
        assert torch.equal(o1[0], out[r]) and torch.equal(s1[0], sh[r])
    og, sg = torch.empty_like(out), torch.empty_like(sh)
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        G.routed2(x, pk, wt, L, s, out=og, out_shared=sg)
    torch.cuda.current_stream().wait_stream(st)
    gph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gph):
        G.routed2(x, pk, wt, L, s, out=og, out_shared=sg)
    og.zero_()
    gph.replay()
    torch.cuda.synchronize()
    assert torch.equal(og, out) and torch.equal(sg, sh)


def test_skipped_picks_and_empty_rows(dev, small_moe):
    """Picks outside [0, E) are skipped (the reference's rule); a row whose routed picks are all skipped gets a zero
    routed sum and keeps its shared-expert output; the other rows are unchanged bit for bit."""
    experts_np, xb, pick, wts, gate_w, L = small_moe
    R, k = pick.shape
    s = G.scratch(L, 32, k + 1, dev)
    x = bf(xb, dev)
    pk, wt = torch.from_numpy(pick).to(dev), torch.from_numpy(wts).to(dev)
    out, sh = G.routed2(x, pk, wt, L, s)
    out, sh = out.clone(), sh.clone()
    pk2 = pk.clone()
    pk2[1, :] = -1                                   # row 1: every routed pick skipped
    pk2[2, 0] = C.MOE_E + 5                          # row 2: one pick out of range
    o2, s2 = G.routed2(x, pk2, wt, L, s)
    torch.cuda.synchronize()
    assert torch.equal(o2[0], out[0]) and torch.equal(o2[3], out[3])
    assert bool((o2[1] == 0).all()) and torch.equal(s2[1], sh[1])
    routed, _ = _oracle_moe(experts_np, xb[2:3], pick[2:3, 1:], wts[2:3, 1:], gate_w, k - 1)
    e = rel_err(f32(o2[2:3]), routed)
    assert e < 1e-2, f"row with a skipped pick: max rel err {e:.3e}"
    assert _lib.device_status() == 0
    assert int(s.cnt_gu.abs().sum()) == 0 and int(s.cnt_d.abs().sum()) == 0


def test_empty_calls_return_ok(dev):
    lib = _lib.lib()
    null = None
    assert lib.esp_rot_in(16, 1, 2048, 16, 16, 16, 16, 16, 0, 2048, 9, 256, null) == 0   # rows = 0: nothing to do
    assert lib.esp_combine(16, 16, 16, 0, 2048, 9, null) == 0
    assert lib.esp_ep_combine(16, 16, 16, 16, null, 1, 0, 2048, 9, 8, 256, 2, 0, null) == 0


@functools.lru_cache(maxsize=2)
def _config3_layer(dev, seed=0):
    """256 routed experts 2048 -> 512 -> 2048 with widths 1/2/3 bits (p = .3/.5/.2; 1-2 bit E2M1,
    3 bit int5) and one 4-bit int6 shared expert; router bf16 [256, 2048] N(0, 1/sqrt(2048)); shared gate [2048]."""
    r = C.rng("cfg3", seed)
    D, I, E = 2048, 512, 256
    ex_np = []
    for e in range(E + 1):
        if e == E:
            cb, K = 7, 4
        else:
            bits = int(r.choice([1, 2, 3], p=[0.3, 0.5, 0.2]))
            cb, K = (3, bits) if bits < 3 else (6, 3)
        ex = {}
        for p, (kin, n) in (("gate", (D, I)), ("up", (D, I)), ("down", (I, D))):
            ex[p] = (C.trellis(("cfg3", e, p), kin, n, K), K, cb, C.suh(("cfg3", e, p), kin), C.svh(("cfg3", e, p), n))
        ex_np.append(ex)
    gate = C.bf16_bits((r.standard_normal((E, D)) / np.sqrt(D)).astype(np.float32))
    sgate = C.bf16_bits((r.standard_normal(D) / np.sqrt(D)).astype(np.float32))
    return ex_np, gate, sgate


@pytest.mark.parametrize("R", [1, 3, 8, 32])
def test_config3_layer_with_fused_routing(dev, R):
    ex_np, gate_b, sgate_b = _config3_layer(dev)
    mats = build(ex_np, dev)
    L = G.prepare(mats[:-1], mats[-1], bf(sgate_b, dev))
    k = 8
    s = G.scratch(L, 32, k + 1, dev)
    xb = C.activations(("cfg3-x", R), R, 2048)
    x = bf(xb, dev)
    G.route(x, bf(gate_b, dev), k, L, s)
    out, sh = G.routed2(x, None, None, L, s, k=k)
    torch.cuda.synchronize()
    pick, wts, _ = O.route(xb, gate_b, k, sgate_b, 256)
    P = R * (k + 1)
    assert np.array_equal(s.pick[:P].cpu().numpy().reshape(R, k + 1), pick)
    routed, shared, _ = O.moe(C.bf16_to_f32(xb), pick, s.wts[:P].cpu().numpy().reshape(R, k + 1), ex_np, k)
    for got, want in ((out, routed), (sh, shared)):
        e = rel_err(f32(got), want)
        fl = rel_err(C.bf16_to_f32(C.bf16_bits(want)), want)
        assert e < 1e-2 and e < fl + 2e-3, f"max rel err {e:.3e} (floor {fl:.3e})"
    assert _lib.device_status() == 0
    assert int(s.cnt_layer.abs().sum()) == 0


@pytest.mark.parametrize("R", [1, 5, 32])
def test_one_launch_layer_equals_two_launches(dev, monkeypatch, R):
    """The one-launch layer (gate/up, SwiGLU, down and the per-row combine in one persistent kernel, ready flags
    between the phases) gives the two-launch pipeline's bits, and leaves its counters and flags zero."""
    ex_np, gate_b, sgate_b = _config3_layer(dev, seed=1)
    mats = build(ex_np, dev)
    L = G.prepare(mats[:-1], mats[-1], bf(sgate_b, dev))
    k = 8
    s = G.scratch(L, 32, k + 1, dev)
    x = bf(C.activations(("one-launch", R), R, 2048), dev)
    G.route(x, bf(gate_b, dev), k, L, s)
    monkeypatch.setattr(G, "MOE_ONE_LAUNCH", False)
    a, b = G.routed2(x, None, None, L, s, k=k)
    a, b = a.clone(), b.clone()
    monkeypatch.setattr(G, "MOE_ONE_LAUNCH", True)
    for _ in range(3):                               # repeated: flags and counters must come back to zero
        o, sh = G.routed2(x, None, None, L, s, k=k)
        torch.cuda.synchronize()
        assert torch.equal(o, a) and torch.equal(sh, b)
    assert _lib.device_status() == 0
    assert int(s.cnt_layer.abs().sum()) == 0


@pytest.mark.parametrize("R", [1, 8, 32])
def test_route_with_rotation_equals_route_then_rot_in(dev, R):
    """The routing launch's folded input rotation (esp_route_rot) writes exactly rot_in's xg / xu, and the same picks,
    weights and grouping as esp_route_group; its counters come back to zero."""
    ex_np, gate_b, sgate_b = _config3_layer(dev)
    mats = build(ex_np, dev)
    L = G.prepare(mats[:-1], mats[-1], bf(sgate_b, dev))
    k = 8
    s = G.scratch(L, 32, k + 1, dev)
    x = bf(C.activations(("route-rot", R), R, 2048), dev)
    gate = bf(gate_b, dev)
    P = R * (k + 1)
    G.route(x, gate, k, L, s)                     # routing with the folded rotation
    torch.cuda.synchronize()
    got = [t[:P].clone() for t in (s.xg, s.xu, s.pick, s.wts)] + [s.count.clone()]
    s.rotated = False
    s.xg.zero_()
    s.xu.zero_()
    ids, members = s.window(R)
    _lib.ext().route_group(x, gate, L.gate_w, k, L.shared_id, s.logits, s.route_counter, s.pick[:P], s.wts[:P], ids,
                           s.count, members)
    _lib.ext().rot_in(x, x.stride(0), s.pick[:P], L.gate.suh, L.up.suh, s.xg, s.xu, R, 2048, k + 1, L.E)
    torch.cuda.synchronize()
    want = [t[:P] for t in (s.xg, s.xu, s.pick, s.wts)] + [s.count]
    for a, b in zip(got, want):
        assert torch.equal(a, b)
    assert int(s.route_counter.abs().sum()) == 0
    assert _lib.device_status() == 0
