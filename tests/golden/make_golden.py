"""Generate tests/golden/golden.npz by running the REFERENCE plugin's own CUDA extension on a GPU.

The extension is the reference's csrc/ built from its sources by oracle/build_ref.py into oracle/_ref/ (test
infrastructure; nothing of it is committed). This script calls its functions (dequant, had, dense, route_group,
group_shared, rot_in, grouped, gateup_epilogue, down_combine2) with the deterministic inputs of cases.py, using the host
parameters the reference's own Python layer would pass (dense.plan, experts.tile_config restated below), and stores
the outputs. The CPU oracle is then pinned against these outputs by tests/test_golden.py (no GPU needed).

usage (on a GPU box): python tests/golden/make_golden.py [--so oracle/_ref/espalier_ref_ext.so]
"""
from __future__ import annotations

import argparse
import importlib.machinery
import importlib.util
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(ROOT / "oracle"))
import cases as C  # noqa: E402
import oracle as O  # noqa: E402


def load_ref(path: Path):
    loader = importlib.machinery.ExtensionFileLoader("espalier_ref_ext", str(path))
    spec = importlib.util.spec_from_loader("espalier_ref_ext", loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def ref_plan(K: int, N: int, sms: int):
    """The reference's shape-only dense tiling (vllm_espalier/dense.py:22-39), restated."""
    nb, kt = N // 128, K // 16
    if nb >= 8 * sms:
        return 1, 4, 1
    if 2 * nb >= 3 * sms and kt % (8 * 2) == 0:
        return 1, 8, 1
    w, sk = 4, 1
    while nb * sk < 2 * sms and kt % (2 * sk * w) == 0 and kt // (2 * sk * w) >= 2:
        sk *= 2
    return sk, w, 1


def ref_tile_config(K: int, N: int, gateup: bool):
    """vllm_espalier/experts.py:59-68, restated."""
    cands = [(4, 4, 4, 2) if gateup else (4, 4, 1, 2), (8, 4, 4, 1) if gateup else (8, 4, 1, 1), (8, 4, 2, 1),
             (8, 4, 1, 1), (4, 4, 2, 2), (4, 4, 1, 2)]
    for nt, w, sk, pf in cands:
        if K % (16 * sk * w) == 0 and N % (16 * nt) == 0:
            return nt, w, sk, pf
    raise ValueError((K, N))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--so", type=Path, default=ROOT / "oracle" / "_ref" / "espalier_ref_ext.so")
    ap.add_argument("--out", type=Path, default=HERE / "golden.npz")
    a = ap.parse_args()
    ext = load_ref(a.so)
    dev = torch.device("cuda")
    out: dict[str, np.ndarray] = {}
    T16 = lambda a_: torch.from_numpy(np.ascontiguousarray(a_)).to(dev)  # noqa: E731

    # 1. dequant for every compiled (codebook, width) pair
    for cb, k2 in C.COMPILED:
        t = C.dequant_case(cb, k2)
        w = torch.empty((t.shape[0] * 16, t.shape[1] * 16), dtype=torch.float16, device=dev)
        ext.dequant(T16(t), w, k2, cb)
        out[f"dq_{cb}_{k2}"] = w.cpu().numpy().view(np.uint16)
        out[f"dq_{cb}_{k2}_in"] = np.array(C.checksum(t))

    # 2. full state -> value tables
    for cb, k2 in C.TABLE_CASES.items():
        tab = np.zeros(65536, np.uint16)
        seen = np.zeros(65536, bool)
        attempt = 0
        while not seen.all() and attempt < 8:
            t = C.table_trellis(cb, k2, attempt)
            w = torch.empty((t.shape[0] * 16, t.shape[1] * 16), dtype=torch.float16, device=dev)
            ext.dequant(T16(t), w, k2, cb)
            W = w.cpu().numpy().view(np.uint16).ravel()
            S = O.states(t, k2 // 2).ravel()
            if seen[S].any():
                assert (tab[S][seen[S]] == W[seen[S]]).all(), "one state decoded to two values"
            tab[S] = W
            seen[S] = True
            attempt += 1
        assert seen.all(), f"codebook {cb}: {int((~seen).sum())} states never drawn"
        out[f"table_{cb}"] = tab

    # 3. had
    x, pre, post = C.had_case()
    y = torch.empty(x.shape, dtype=torch.float16, device=dev)
    ext.had(T16(x), T16(pre), T16(post), y)
    out["had_pre_post"] = y.cpu().numpy().view(np.uint16)
    ext.had(T16(x), T16(pre), None, y)
    out["had_pre"] = y.cpu().numpy().view(np.uint16)

    # 4. dense layers through the reference's fused dense kernel
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    for name, K, Ns, cb, k2, Ms, xdt in C.DENSE_CASES:
        for M in Ms:
            mats, xf = C.dense_inputs(name, K, Ns, cb, k2, M, xdt)
            tdt = torch.bfloat16 if xdt == "bf16" else torch.float16
            xt = torch.from_numpy(xf).to(dev).to(tdt)
            N = sum(Ns)
            sk, w, pf = ref_plan(K, N, sms)
            y = torch.empty((M, N), dtype=tdt, device=dev)
            Z = torch.empty(max(sk * 32 * N, 1), dtype=torch.float32, device=dev)
            xh = torch.empty(4 * 32 * K, dtype=torch.float16, device=dev)
            cnt = torch.zeros(2 * N // 128, dtype=torch.int32, device=dev)
            col0, c = [], 0
            for n in Ns:
                col0.append(c)
                c += n
            ext.dense(xt, [T16(m[0]) for m in mats], [T16(m[1]) for m in mats], [T16(m[2]) for m in mats], col0, y,
                      xh, Z, cnt, k2, cb, sk, w, pf, 32 * 1024)
            out[f"dense_{name}_{M}"] = y.cpu().view(torch.int16).numpy().view(np.uint16)
            out[f"dense_{name}_{M}_in"] = np.array(C.checksum(xf, *[m[0] for m in mats]))

    # 5. fused routing (the reference's route_group: fp32 logits, bf16-rounded, softmax/top-k, grouping)
    xb, gb, sb = C.route_inputs()
    tb = lambda b: torch.from_numpy(b.view(np.int16)).to(dev).view(torch.bfloat16)  # noqa: E731
    R, E, k = C.ROUTE_R, C.ROUTE_E, C.ROUTE_K
    slots = k + 1
    logits = torch.zeros(R * (E + 1), dtype=torch.float32, device=dev)
    counter = torch.zeros(1, dtype=torch.int32, device=dev)
    pick = torch.zeros(R * slots, dtype=torch.int32, device=dev)
    wts = torch.zeros(R * slots, dtype=torch.float32, device=dev)
    maxu = min(R * slots, E + 1)
    uids = torch.zeros(maxu, dtype=torch.int32, device=dev)
    ucount = torch.zeros(1, dtype=torch.int32, device=dev)
    members = torch.full((maxu, R), -1, dtype=torch.int32, device=dev)
    ext.route_group(tb(xb), tb(gb), tb(sb), k, E, logits, counter, pick, wts, uids, ucount, members)
    n = int(ucount.item())
    out["route_pick"] = pick.cpu().numpy().reshape(R, slots)
    out["route_wts"] = wts.cpu().numpy().reshape(R, slots)
    out["route_logits"] = logits.cpu().numpy().reshape(R, E + 1)
    out["route_uids"] = uids[:n].cpu().numpy()
    out["route_members"] = members[:n].cpu().numpy()

    # 6. a small MoE layer through the reference's routed2 launch sequence (experts.py:231-261)
    experts, xb, pick_np, wts_np, gate_w = C.moe_inputs()
    Etot = len(experts)
    D, I, Rm, km = C.MOE_D, C.MOE_I, C.MOE_R, C.MOE_K
    slots = km + 1
    P = Rm * slots
    xt = tb(xb)

    def tables(p):
        ptr = torch.tensor([0] * Etot, dtype=torch.int64)
        keep = []
        for e, ex in enumerate(experts):
            tt = T16(ex[p][0])
            keep.append(tt)
            ptr[e] = tt.data_ptr()
        k2s = torch.tensor([2 * ex[p][1] for ex in experts], dtype=torch.int32, device=dev)
        cbs = torch.tensor([ex[p][2] for ex in experts], dtype=torch.int32, device=dev)
        return ptr.to(dev), k2s, cbs, keep

    def stack(p, j):
        return torch.stack([T16(ex[p][j]) for ex in experts]).contiguous()

    gp, gk, gc, keep_g = tables("gate")
    upp, uk, uc, keep_u = tables("up")
    dp, dk, dc, keep_d = tables("down")
    suh_g, suh_u, svh_g, svh_u = stack("gate", 3), stack("up", 3), stack("gate", 4), stack("up", 4)
    suh_d, svh_d = stack("down", 3), stack("down", 4)
    cfg_gu, cfg_d = ref_tile_config(D, I, True), ref_tile_config(I, D, False)
    xg = torch.zeros((P, D), dtype=torch.float16, device=dev)
    xu = torch.zeros((P, D), dtype=torch.float16, device=dev)
    xd = torch.zeros((P, I), dtype=torch.float16, device=dev)
    z = torch.zeros((max(2 * cfg_gu[2] * I, cfg_d[2] * D) * P,), dtype=torch.float32, device=dev)
    yb = torch.zeros((P, D), dtype=torch.float32, device=dev)
    pk = torch.zeros(P, dtype=torch.int32, device=dev)
    wt = torch.zeros(P, dtype=torch.float32, device=dev)
    maxu = min(P, Etot)
    ids = torch.zeros(maxu, dtype=torch.int32, device=dev)
    cnt = torch.zeros(1, dtype=torch.int32, device=dev)
    mem = torch.full((maxu, Rm), -1, dtype=torch.int32, device=dev)
    ext.group_shared(T16(pick_np), T16(wts_np), xt, xt.stride(0), tb(gate_w), Etot - 1, pk, wt, ids, cnt, mem, Rm, km,
                     Etot)
    ext.rot_in(xt, xt.stride(0), pk, suh_g, suh_u, xg, xu, Rm, D, slots, Etot)
    nt, w, sk, pf = cfg_gu
    lo = min(int(gk.min()), int(uk.min()))
    hi = max(int(gk.max()), int(uk.max()))
    ext.grouped(xg, xu, gp, upp, gk, uk, gc, uc, ids, cnt, mem, z, 2, D, I, P, sk, slots, nt, w, pf, lo, hi)
    ext.gateup_epilogue(z, pk, svh_g, svh_u, suh_d, xd, Rm, P, I, sk, slots, Etot, math.inf, 1)
    nt, w, sk, pf = cfg_d
    ext.grouped(xd, xd, dp, dp, dk, dk, dc, dc, ids, cnt, mem, z, 1, I, D, P, sk, slots, nt, w, pf, int(dk.min()),
                int(dk.max()))
    o = torch.empty((Rm, D), dtype=torch.bfloat16, device=dev)
    osh = torch.empty((Rm, D), dtype=torch.bfloat16, device=dev)
    ext.down_combine2(z, pk, svh_d, yb, wt, o, osh, Rm, P, D, sk, slots, Etot, km)
    torch.cuda.synchronize()
    out["moe_out"] = o.cpu().view(torch.int16).numpy().view(np.uint16)
    out["moe_shared"] = osh.cpu().view(torch.int16).numpy().view(np.uint16)
    out["moe_xd"] = xd.cpu().numpy().view(np.uint16)
    out["moe_pick"] = pk.cpu().numpy().reshape(Rm, slots)
    out["moe_wts"] = wt.cpu().numpy().reshape(Rm, slots)
    out["moe_y"] = yb.cpu().numpy().reshape(Rm, slots, D)
    out["meta_device"] = np.array(torch.cuda.get_device_name())
    np.savez_compressed(a.out, **out)
    print(f"wrote {a.out} ({len(out)} arrays)")


if __name__ == "__main__":
    main()
