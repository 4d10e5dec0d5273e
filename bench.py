"""Benchmark of the Espalier B200 decode hot path (one JSON line on rank 0).

Headline ("fused dense decode of one attention/DeltaNet-style block, hidden 2048"): a step is
one decode step through L = 40 synthetic blocks of q/k/v (2048 -> 4096 + 512 + 512, one fused launch) and o
(4096 -> 2048), 4-bit trellis with the int5 codebook, random-init seeded weights; block i's o output is block i+1's
input (q stands in for the attention output). 40 blocks hold 379 MB of compressed weights, 3x the 126 MB L2, so every
step streams its weights from HBM (no flush needed). Steps are captured once in a CUDA graph and replayed.

  value        decode tok/s at batch 1 (whole job: all ranks' tokens / the slowest rank's time)
  batches      the same at batch 1 / 8 / 32, with compressed-weight GB/s and % of the measured HBM peak
  roofline     HBM roofline of the fused dense decode kernel on algorithmic (compressed) bytes
  e2e          the same metric through the public API with host (pinned) input and output copied every step
  cpu_baseline the reference's decode-then-matmul path restated on the host cores (oracle), bounded sample
  config1      BASELINE configs[0]: one 2048 -> 4096 int6 4-bit layer at batch 1, with its CPU path timed beside it
  moe          BASELINE configs[2]: a stack of MoE layers at batch 1 / 8 / 32 (expert parallel under torchrun, with
               every rank's output compared bit for bit with the one-GPU layer)
  route        BASELINE configs[3]: the fused routing kernel alone, 5% near-tied rows, ids checked against exact
               routing (fp64 logits rounded once to bf16, lowest id on ties) in the same run
  decoder      BASELINE configs[4]: the 40-layer synthetic decoder, batch 1 / 8 / 32 and the 4-token MTP-3
               verification batch, with a roofline and a time split by kernel class at batch 1

N > 1 (torchrun): the dense path runs as data-parallel replicas (no collective on the data path); the MoE stack runs
expert parallel (`ep_headline`).
--impl reference: the reference's CPU path (the C oracle's decode + torch) as the headline arm, plus `ref_kernels`: the
reference's own CUDA kernels (built from its sources into oracle/_ref) timed on the same workloads.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HIDDEN, Q, KV, O_IN = 2048, 4096, 512, 4096
QKV_N = [Q, KV, KV]
BITS, GRID, KCB = 4, 3, 6            # 4-bit, esp_grid code 3 = int5, kernel codebook 6
MOE_D, MOE_I, MOE_E, MOE_K = 2048, 512, 256, 8
VOCAB = 248320
RES_SCALE = 0.1


def block_bytes() -> int:
    """Algorithmic bytes of one block: trellis + suh + svh of q, k, v and o (9,472,000 for the 4-bit config-2 block)."""
    qkv = HIDDEN * sum(QKV_N) * BITS // 8 + 3 * HIDDEN * 2 + sum(QKV_N) * 2
    o = O_IN * HIDDEN * BITS // 8 + O_IN * 2 + HIDDEN * 2
    return qkv + o


# ---------------------------------------------------------------------------------------------------------------
# synthetic coded matrices (torch only: both arms build the same weights from the same seeds)
# ---------------------------------------------------------------------------------------------------------------
class Mat:
    """A random coded matrix: uniform int16 trellis, +-1 suh, +-U(0.5, 1.5)/64 svh (the synthetic stand-in for a checkpoint)."""

    def __init__(self, kin, n, K, grid, gen, dev):
        self.trellis = torch.randint(-32768, 32768, (kin // 16, n // 16, 16 * K), dtype=torch.int16, device=dev,
                                     generator=gen)
        self.suh = (torch.randint(0, 2, (kin,), device=dev, generator=gen) * 2 - 1).half()
        self.svh = ((torch.randint(0, 2, (n,), device=dev, generator=gen) * 2 - 1).float() *
                    (0.5 + torch.rand(n, device=dev, generator=gen)) / 64).half()
        self.K, self.cb, self.in_features, self.out_features = K, grid, kin, n


def mat_bytes(m) -> int:
    return m.trellis.numel() * 2 + m.suh.numel() * 2 + m.svh.numel() * 2


def make_blocks(layers: int, dev, seed: int = 0):
    """[(q/k/v matrices, o matrix)] of config 2."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    return [([Mat(HIDDEN, n, BITS, GRID, gen, dev) for n in QKV_N], Mat(O_IN, HIDDEN, BITS, GRID, gen, dev))
            for _ in range(layers)]


def make_moe(layers: int, dev, seed: int = 1):
    """Config-3 layers: [dict(ex=[(gate, up, down)] * 256, sh=(gate, up, down), gate_w, gate)]. Widths 1/2/3 bits at
    p = .3/.5/.2 (1-2 bit E2M1, 3 bit int5), a 4-bit int6 shared expert, router bf16 [256, 2048] and shared gate
    [2048] N(0, 1/2048). Every rank draws every expert, so all ranks hold the same weights."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    rng = np.random.default_rng(seed)
    out = []
    for i in range(layers):
        ex = []
        for e in range(MOE_E):
            bits = int(rng.choice([1, 2, 3], p=[0.3, 0.5, 0.2]))
            K, grid = (bits, 1) if bits < 3 else (3, 3)          # esp grid codes: 1 = E2M1, 3 = int5
            ex.append((Mat(MOE_D, MOE_I, K, grid, gen, dev), Mat(MOE_D, MOE_I, K, grid, gen, dev),
                       Mat(MOE_I, MOE_D, K, grid, gen, dev)))
        sh = (Mat(MOE_D, MOE_I, 4, 4, gen, dev), Mat(MOE_D, MOE_I, 4, 4, gen, dev), Mat(MOE_I, MOE_D, 4, 4, gen, dev))
        gw = torch.Generator(device=dev)
        gw.manual_seed(seed * 1000 + i)                       # the replicated router: the same on every rank
        gate_w = (torch.randn(MOE_D, device=dev, generator=gw) / math.sqrt(MOE_D)).to(torch.bfloat16)
        gate = (torch.randn(MOE_E, MOE_D, device=dev, generator=gw) / math.sqrt(MOE_D)).to(torch.bfloat16)
        out.append({"ex": ex, "sh": sh, "gate_w": gate_w, "gate": gate})
    return out


def rows_for(R: int, dim: int, dev, seed: int) -> torch.Tensor:
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return torch.randn(R, dim, device=dev, generator=g).to(torch.bfloat16)


class Graphed:
    """A step with static buffers: eager() once, capture() into a CUDA graph, __call__ replays it."""
    graph = None

    def capture(self):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self.eager()
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.eager()

    def __call__(self):
        self.graph.replay() if self.graph is not None else self.eager()


class Step(Graphed):
    """One decode step through the dense blocks at batch R. `blocks` = [(qkv, o)] objects with forward(x, out=)."""

    def __init__(self, blocks, R, dev):
        self.blocks, self.R = blocks, R
        self.x = rows_for(R, HIDDEN, dev, 11)
        self.ys = [(torch.empty(R, sum(QKV_N), dtype=torch.bfloat16, device=dev),
                    torch.empty(R, HIDDEN, dtype=torch.bfloat16, device=dev)) for _ in blocks]

    @property
    def out(self):
        return self.ys[-1][1]

    def eager(self):
        x = self.x
        for (qkv, o), (yq, yo) in zip(self.blocks, self.ys):
            qkv.forward(x, out=yq)
            o.forward(yq[:, :O_IN], out=yo)
            x = yo

    def launches(self) -> int:
        # per block and matrix set (qkv, o): one decode launch with the input rotation fused up to 8 rows, a rotation
        # launch plus the decode launch above
        return (2 if self.R <= 8 else 4) * len(self.blocks)


def our_blocks(raw):
    from vllm_espalier_b200 import dense as D
    return [(D.Dense(qkv), D.Dense([o])) for qkv, o in raw]


class Clocks:
    """nvidia-smi samples of SM clock and throttle reasons while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "100", "-i", str(gpu_index)], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.p.terminate()
        self.p.wait()
        self.f.seek(0)
        rows = [r.split(", ") for r in self.f.read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip() == "Active"})
        busy = [v for v in sm if v > 0]
        return {"sm_mhz": statistics.median(busy) if busy else None, "sm_max_mhz": float(rows[0][2]),
                "reasons": reasons, "samples": len(rows)}


def time_steps(step, steps: int, warmup: int, dist, dev) -> float:
    """ms a step: CUDA events on the launching stream around `steps` replays after `warmup`, max over ranks."""
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        step()
    b.record()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ms = a.elapsed_time(b) / steps
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def time_e2e(step: Step, steps: int, warmup: int, dist, dev) -> tuple[float, int, int]:
    """Host input copied in (pinned, async) and the step's output read back, every step, inside the timed region."""
    xh = torch.empty_like(step.x, device="cpu").pin_memory()
    xh.copy_(step.x.cpu())
    oh = torch.empty_like(step.out, device="cpu").pin_memory()

    def one():
        step.x.copy_(xh, non_blocking=True)
        step()
        oh.copy_(step.out, non_blocking=True)
    ms = time_steps(one, steps, warmup, dist, dev)
    return ms, xh.numel() * xh.element_size(), oh.numel() * oh.element_size()


# ---------------------------------------------------------------------------------------------------------------
# MoE layers (config 3), one GPU or expert parallel
# ---------------------------------------------------------------------------------------------------------------
class MoEStep(Graphed):
    """One decode step through MoE layers at batch R: [(layer, gate)] where layer is an experts.Layer (route +
    routed2) or an ep.EPLayer (its forward)."""

    def __init__(self, G, layers, R, dev, seed: int = 21):
        self.G, self.layers, self.R = G, layers, R
        self.x = rows_for(R, MOE_D, dev, seed)
        self.s = G.scratch(layers[0][0], 32, MOE_K + 1, dev) if isinstance(layers[0][0], G.Layer) else None
        self.outs = [(torch.empty(R, MOE_D, dtype=torch.bfloat16, device=dev),
                      torch.empty(R, MOE_D, dtype=torch.bfloat16, device=dev)) for _ in layers]

    def eager(self):
        for (L, gate), (o, so) in zip(self.layers, self.outs):
            if self.s is not None:
                self.G.route(self.x, gate, MOE_K, L, self.s)
                self.G.routed2(self.x, None, None, L, self.s, out=o, out_shared=so, k=MOE_K)
            else:
                L.forward(self.x, gate, out=o, out_shared=so)


def touched_bytes(G, layers, raw, x, dev) -> tuple[int, list[int]]:
    """Compressed bytes one step at rows x reads on one GPU: each layer's router and the matrices of every expert its
    routing picked; and the distinct experts a layer."""
    total, distinct = 0, []
    for (L, gate), r in zip(layers, raw):
        s = G.scratch(L, 32, MOE_K + 1, dev)
        G.route(x, gate, MOE_K, L, s)
        torch.cuda.synchronize()
        n = int(s.count[0].item())
        ids, _ = s.window(x.shape[0])
        distinct.append(n)
        for e in ids[:n].tolist():
            total += sum(mat_bytes(m) for m in (r["sh"] if e == L.shared_id else r["ex"][e]))
        total += gate.numel() * 2 + L.gate_w.numel() * 2
    return total, distinct


def moe_bench(dev, layers: int, steps: int, warmup: int, dist, peak: float, rank: int = 0, world: int = 1) -> dict:
    from vllm_espalier_b200 import ep as EP
    from vllm_espalier_b200 import experts as G
    from vllm_espalier_b200._env import MOE_ONE_LAUNCH as one
    raw = make_moe(layers, dev)
    full = [(G.prepare(r["ex"], r["sh"], r["gate_w"]), r["gate"]) for r in raw]     # every expert (one GPU's layer)
    if world > 1:
        e0, e1 = EP.expert_range(rank, world, MOE_E)
        run = [(EP.EPLayer(r["ex"][e0:e1], r["sh"], r["gate_w"], rank, world, MOE_E, rows=32, k=MOE_K), r["gate"])
               for r in raw]
    else:
        run = full
    res = {}
    for R in (1, 8, 32):
        st = MoEStep(G, run, R, dev, seed=21 + 1000 * rank)
        st.eager()
        st.capture()
        ms = time_steps(st, steps, warmup, dist, dev)
        st.graph = None
        entry = {"us_per_layer": ms * 1e3 / layers, "tok_s_layer_stack": world * R / (ms * 1e-3)}
        nbytes, distinct = touched_bytes(G, full, raw, st.x, dev)
        gbs = nbytes / (ms * 1e-3) / 1e9
        entry.update({"touched_mb_per_layer": nbytes / layers / 1e6, "distinct_experts_per_layer":
                      sum(distinct) / layers, "weight_gbs": gbs, "hbm_frac": gbs / peak})
        if world > 1:
            # the same rows through the one-GPU layer holding every expert: the EP outputs must be identical
            st.eager()
            same = True
            s = G.scratch(full[0][0], 32, MOE_K + 1, dev)
            for (L, gate), (o, so) in zip(full, st.outs):
                G.route(st.x, gate, MOE_K, L, s)
                want, want_sh = G.routed2(st.x, None, None, L, s, k=MOE_K)
                same &= bool(torch.equal(o, want)) and bool(torch.equal(so, want_sh))
            flag = torch.tensor([1 if same else 0], device=dev)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            entry["ep_bitwise"] = bool(flag.item())
            entry["weight_gbs_note"] = ("bytes the rank's rows pick on one GPU over the slowest rank's time; each "
                                        "rank reads only its own experts' share")
        res[str(R)] = entry
    from vllm_espalier_b200._env import EP_EXCHANGE
    exch = ("peer stores of rows and picks into the owners' inboxes (CUDA IPC, release/acquire flags), local "
            "experts, peer stores of per-slot rows back to their home ranks" if EP_EXCHANGE == "p2p" else
            "NCCL all_to_all dispatch of rows and picks, local experts, all_to_all of per-slot rows back")
    how = (f"routing with the experts' input rotation fused, then "
           f"{'one fused expert launch' if one else 'two fused expert launches'} a layer"
           if world == 1 else f"expert parallel over {world} GPUs: local routing, {exch}, slot-ordered combine")
    return {"workload": f"BASELINE configs[2]: {layers} MoE layers a step, each with its own experts and router "
                        f"(256 experts 1/2/3-bit E2M1/int5, int6 shared, top-8), {how}, graph replay; at batch 1 the "
                        f"step touches more than the L2 holds",
            "layers": layers, "world": world, "scaling": "weak (R rows a rank)" if world > 1 else None,
            "launches_per_layer": (2 if one else 3) if world == 1 else None, "batches": res}


# ---------------------------------------------------------------------------------------------------------------
# routing microbench (config 4)
# ---------------------------------------------------------------------------------------------------------------
ROUTE_COPIES = 150                     # router copies a replay walks through: 157 MB, more than the L2


def bf16_round_f64(v: np.ndarray) -> np.ndarray:
    """float64 -> the nearest bf16 value (ties to even), as float32: one rounding, no fp32 step."""
    b = np.ascontiguousarray(v, dtype=np.float64).view(np.uint64)
    lsb = (b >> np.uint64(45)) & np.uint64(1)
    b = (b + np.uint64((1 << 44) - 1) + lsb) & ~np.uint64((1 << 45) - 1)
    return b.view(np.float64).astype(np.float32)


def exact_top_k(x: torch.Tensor, gate: torch.Tensor, k: int) -> np.ndarray:
    """Exact routing (the reference's tests/gpu_route.py:89 definition): fp64 logits of the bf16 inputs rounded once
    to bf16, the k largest, lowest id first on ties."""
    lg = bf16_round_f64(x.double().cpu().numpy() @ gate.double().cpu().numpy().T)
    ids = np.arange(lg.shape[1])
    return np.stack([np.lexsort((ids, -row))[:k] for row in lg]).astype(np.int32)


def near_tie_rows(R: int, gate: torch.Tensor, k: int, dev, seed: int, frac: float = 0.05) -> torch.Tensor:
    """bf16 rows N(0, 1) where a `frac` share (at least one) is moved along w_a - w_b so that the fp64 logit gap
    between ranks k and k + 1 is below 1e-3."""
    r = np.random.default_rng(seed)
    x = rows_for(R, MOE_D, dev, seed).double().cpu().numpy()
    g = gate.double().cpu().numpy()
    for i in r.choice(R, max(1, int(frac * R)), replace=False):
        lg = g @ x[i]
        order = np.argsort(-lg)
        d = g[order[k - 1]] - g[order[k]]
        x[i] = x[i] - d * (lg[order[k - 1]] - lg[order[k]] - r.uniform(-5e-4, 5e-4)) / (d @ d)
    return torch.from_numpy(x).float().to(torch.bfloat16).to(dev)


def route_inputs(dev):
    gw = torch.Generator(device=dev)
    gw.manual_seed(4001)
    gate = (torch.randn(MOE_E, MOE_D, device=dev, generator=gw) / math.sqrt(MOE_D)).to(torch.bfloat16)
    sgate = (torch.randn(MOE_D, device=dev, generator=gw) / math.sqrt(MOE_D)).to(torch.bfloat16)
    return gate, sgate, [gate.clone() for _ in range(ROUTE_COPIES)]


class RouteStep(Graphed):
    def __init__(self, call, copies, x):
        self.call, self.copies, self.x = call, copies, x

    def eager(self):
        for g in self.copies:
            self.call(self.x, g)


def route_bench(dev, steps: int, warmup: int, dist, call, picks) -> dict:
    """call(x, gate) routes x with router `gate` into scratch; picks(R) reads back the routed ids [R, 8]."""
    gate, sgate, copies = route_inputs(dev)
    res = {}
    for R in (1, 8, 32):
        x = near_tie_rows(R, gate, MOE_K, dev, seed=4100 + R)
        call(x, gate)
        torch.cuda.synchronize()
        got = picks(R)
        want = exact_top_k(x, gate, MOE_K)
        st = RouteStep(call, copies, x)
        st.capture()
        ms = time_steps(st, max(steps, 3), warmup, dist, dev)
        st.graph = None
        res[str(R)] = {"us": ms * 1e3 / len(copies), "ids_exact": bool(np.array_equal(got, want)),
                       "near_tie_rows": max(1, int(0.05 * R))}
    return {"workload": f"BASELINE configs[3]: router GEMV bf16 256 x 2048, softmax top-8, renormalised weights, "
                        f"shared-expert gate and grouping, one launch; {ROUTE_COPIES} router copies a replay (cold L2)",
            "batches": res}


def our_route(dev):
    """The fused routing kernel on its own (ext().route_group: GEMV, top-k, renormalisation, shared gate, grouping)."""
    from vllm_espalier_b200 import experts as G
    from vllm_espalier_b200._lib import ext
    gate, sgate, _ = route_inputs(dev)
    s = G.Scratch(MOE_E + 1, MOE_D, MOE_I, 32, MOE_K + 1, dev)

    def call(x, g):
        R = x.shape[0]
        ids, members = s.window(R)
        n = R * s.slots
        ext().route_group(x, g, sgate, MOE_K, MOE_E, s.logits, s.route_counter, s.pick[:n], s.wts[:n], ids, s.count,
                          members)

    def picks(R):
        return s.pick[:R * (MOE_K + 1)].view(R, MOE_K + 1)[:, :MOE_K].cpu().numpy()
    return call, picks


# ---------------------------------------------------------------------------------------------------------------
# config 1: one 2048 -> 4096 int6 4-bit layer at batch 1
# ---------------------------------------------------------------------------------------------------------------
C1_K, C1_N, C1_BITS, C1_GRID, C1_KCB = 2048, 4096, 4, 4, 7
C1_COPIES = 64                          # 4.2 MB each: 269 MB a replay, more than the L2


def config1_bytes() -> int:
    return C1_K * C1_N * C1_BITS // 8 + C1_K * 2 + C1_N * 2


class LayerStep(Graphed):
    def __init__(self, layers, x, n):
        self.layers, self.x = layers, x
        self.ys = [torch.empty(x.shape[0], n, dtype=x.dtype, device=x.device) for _ in layers]

    def eager(self):
        for d, y in zip(self.layers, self.ys):
            d.forward(self.x, out=y)


def config1_mats(dev):
    gen = torch.Generator(device=dev)
    gen.manual_seed(7001)
    return [Mat(C1_K, C1_N, C1_BITS, C1_GRID, gen, dev) for _ in range(C1_COPIES)]


def config1_bench(dev, steps: int, warmup: int, dist, peak: float, cpu_seconds: float | None) -> dict:
    from vllm_espalier_b200 import dense as D
    mats = config1_mats(dev)
    x = rows_for(1, C1_K, dev, 7002)
    st = LayerStep([D.Dense([m]) for m in mats], x, C1_N)
    st.eager()
    st.capture()
    ms = time_steps(st, steps, warmup, dist, dev)
    st.graph = None
    us = ms * 1e3 / C1_COPIES
    gbs = config1_bytes() / (us * 1e-6) / 1e9
    out = {"workload": "BASELINE configs[0]: one 2048 -> 4096 matrix, 4-bit trellis, int6 codebook, batch 1 "
                       f"(fused dense kernel, {C1_COPIES} copies a replay, cold L2)",
           "us_per_call": us, "weight_gbs": gbs, "hbm_frac": gbs / peak, "bytes_per_call": config1_bytes()}
    if cpu_seconds:
        out["cpu"] = cpu_layer(mats[0], x, cpu_seconds)
    return out


# ---------------------------------------------------------------------------------------------------------------
# the reference's decode-then-matmul path on the host cores (the CPU baseline legs)
# ---------------------------------------------------------------------------------------------------------------
def _host_hadamard():
    h = torch.ones(1, 1)
    while h.shape[0] < 128:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    H = h / 128 ** 0.5
    return lambda v: (v.view(*v.shape[:-1], -1, 128) @ H).view(v.shape)


def _cpu_setup():
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    return O, threads


def cpu_layer(m, x: torch.Tensor, seconds: float) -> dict:
    """One matrix through the reference's decode-then-matmul path (vllm_espalier/ops.py:45-51) on the host cores:
    decode W (the C oracle's word-window decode, OpenMP), H(x * suh), x @ W (torch), H(.) * svh."""
    O, threads = _cpu_setup()
    had = _host_hadamard()
    T, su, sv = m.trellis.cpu().numpy(), m.suh.cpu().float(), m.svh.cpu().float()
    xf = x.float().cpu()
    kcb = {0: 1, 1: 3, 3: 6, 4: 7}[m.cb]
    n, dec, t0 = 0, 0.0, time.perf_counter()
    while n < 2 or time.perf_counter() - t0 < seconds:
        td = time.perf_counter()
        W = torch.from_numpy(O.dequant_f32(T, m.K, kcb))
        dec += time.perf_counter() - td
        xh = had(xf * su).half().float()
        _ = (had(xh @ W) * sv).to(torch.bfloat16)
        n += 1
    el = time.perf_counter() - t0
    return {"ms_per_call": el / n * 1e3, "decode_ms_per_call": dec / n * 1e3, "cores": threads, "kind": "port",
            "sample": f"{n} calls in {el:.1f} s"}


def cpu_baseline(raw_blocks, R: int, layers: int, seconds: float = 10.0) -> dict:
    """The reference's decode-then-matmul path (vllm_espalier/ops.py:45-51: decode W, H(x suh), x @ W, H * svh)
    restated on the host: trellis decode by the C oracle's word-window decode straight to fp32 (OpenMP, all cores;
    bit-identical to its bit-serial restatement), matmul by torch on all cores. Timed on a bounded sample of whole
    blocks of this workload, scaled to the step."""
    O, threads = _cpu_setup()
    had = _host_hadamard()
    host = [([(m.trellis.cpu().numpy(), m.suh.cpu().float(), m.svh.cpu().float()) for m in qkv],
             (o.trellis.cpu().numpy(), o.suh.cpu().float(), o.svh.cpu().float())) for qkv, o in raw_blocks]
    x = torch.randn(R, HIDDEN).to(torch.bfloat16).float()
    n_blocks, t0, decode_s = 0, time.perf_counter(), 0.0
    while True:
        for qkv_host, (T, su, sv) in host:
            ys = []
            for Tq, suq, svq in qkv_host:
                td = time.perf_counter()
                W = torch.from_numpy(O.dequant_f32(Tq, BITS, KCB))
                decode_s += time.perf_counter() - td
                xh = had(x * suq).half().float()
                ys.append(had(xh @ W) * svq)
            yq = torch.cat(ys, 1).to(torch.bfloat16).float()
            td = time.perf_counter()
            W = torch.from_numpy(O.dequant_f32(T, BITS, KCB))
            decode_s += time.perf_counter() - td
            xh = had(yq[:, :O_IN] * su).half().float()
            x = (had(xh @ W) * sv).to(torch.bfloat16).float()
            n_blocks += 1
            if time.perf_counter() - t0 > seconds:
                break
        if time.perf_counter() - t0 > seconds:
            break
    el = time.perf_counter() - t0
    per_block = el / n_blocks
    return {"value": R / (per_block * layers), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{n_blocks} q/k/v/o blocks at batch {R} (the step's {layers} blocks in turn; {el:.1f} s, of "
                      f"which trellis decode {decode_s:.1f} s), scaled to one {layers}-block step",
            "block_ms": per_block * 1e3}


# ---------------------------------------------------------------------------------------------------------------
# the full synthetic decoder on one GPU. 40 layers, hidden 2048, each a mixer block (the
# config-2 q/k/v and o projections, 4-bit int5, around a mixer core) and a config-3 MoE layer, with RMSNorms and
# residual adds; 3:1 DeltaNet : gated-attention blocks; bf16 embedding [248320, 2048]; LM head 2048 -> 248320, 6-bit
# mcg. The mixer cores (DeltaNet, attention with an fp8 KV cache, MTP) are not on this path: both sides of a parity
# check use the same stand-in (mixer_core), a fixed elementwise function of the q/k/v projection.
# ---------------------------------------------------------------------------------------------------------------
def rmsnorm(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()).to(torch.bfloat16)


def mixer_core(qkv: torch.Tensor, attention: bool) -> torch.Tensor:
    """Stand-in for the DeltaNet / gated-attention core: [R, 4096 + 512 + 512] -> [R, 4096] bf16."""
    q, k, v = qkv[:, :O_IN].float(), qkv[:, O_IN:O_IN + KV].float(), qkv[:, O_IN + KV:].float()
    kk, vv = k.repeat(1, O_IN // KV), v.repeat(1, O_IN // KV)
    out = q * torch.sigmoid(kk) + vv if attention else torch.tanh(q) * torch.sigmoid(kk) + 0.5 * vv
    return out.to(torch.bfloat16)


def residual(x: torch.Tensor, *ys: torch.Tensor) -> torch.Tensor:
    acc = x.float()
    for y in ys:
        acc = acc + RES_SCALE * y.float()
    return acc.to(torch.bfloat16)


class Decoder:
    """The config-5 decoder through this library's kernels (dense, routing, grouped experts)."""

    def __init__(self, dev, layers: int = 40, seed: int = 2):
        from vllm_espalier_b200 import dense as D
        from vllm_espalier_b200 import experts as G
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        self.layers, self.dev, self.G = layers, dev, G
        raw = make_moe(layers, dev, seed=seed + 1)
        self.moe = [(G.prepare(r["ex"], r["sh"], r["gate_w"]), r["gate"], r["ex"], r["sh"]) for r in raw]
        self.embed = torch.randn(VOCAB, HIDDEN, device=dev, generator=gen).to(torch.bfloat16)
        self.blocks = []
        for i in range(layers):
            qkv = D.Dense([Mat(HIDDEN, n, BITS, GRID, gen, dev) for n in QKV_N])
            o = D.Dense([Mat(O_IN, HIDDEN, BITS, GRID, gen, dev)])
            n1 = (1 + 0.05 * torch.randn(HIDDEN, device=dev, generator=gen)).to(torch.bfloat16)
            n2 = (1 + 0.05 * torch.randn(HIDDEN, device=dev, generator=gen)).to(torch.bfloat16)
            self.blocks.append({"qkv": qkv, "o": o, "n1": n1, "n2": n2, "attention": i % 4 == 3})
        self.final = (1 + 0.05 * torch.randn(HIDDEN, device=dev, generator=gen)).to(torch.bfloat16)
        self.head = D.Dense([Mat(HIDDEN, VOCAB, 6, 0, gen, dev)])   # grid 0 = mcg
        self.s = G.scratch(self.moe[0][0], 32, MOE_K + 1, dev)

    def head_bytes(self) -> int:
        return mat_bytes(self.head.mats[0])

    def layer(self, i: int, x: torch.Tensor, forced=None, picks: list | None = None):
        """Decoder layer i on the residual stream x [R, 2048] bf16 -> (the stream after it, the o projection's output,
        the routed experts' sum, the gated shared expert's output). `forced` = (pick int32 [R, 8], weights fp32
        [R, 8]) replaces the layer's own routing; `picks` collects the routing (pick table with the shared slot)."""
        G, s = self.G, self.s
        blk, (L, gate, _, _) = self.blocks[i], self.moe[i]
        R = x.shape[0]
        h = rmsnorm(x, blk["n1"])
        attn = blk["o"].forward(mixer_core(blk["qkv"].forward(h), blk["attention"]))
        x = residual(x, attn)
        h = rmsnorm(x, blk["n2"])
        if forced is not None:
            out, sh = G.routed2(h, forced[0], forced[1], L, s)
        else:
            G.route(h, gate, MOE_K, L, s)
            out, sh = G.routed2(h, None, None, L, s, k=MOE_K)
        if picks is not None:
            picks.append(s.pick[:R * (MOE_K + 1)].view(R, MOE_K + 1).clone())
        return residual(x, out, sh), attn, out, sh

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        return self.head.forward(rmsnorm(x, self.final))

    def forward(self, tokens: torch.Tensor, picks: list | None = None, forced: list | None = None) -> torch.Tensor:
        """tokens int64 [R] -> logits bf16 [R, VOCAB] (one decode step). `picks` collects each layer's routing;
        `forced` = [(pick, weights)] a layer replaces the layers' own routing."""
        x = self.embed[tokens]
        for i in range(len(self.blocks)):
            x = self.layer(i, x, None if forced is None else forced[i], picks)[0]
        return self.logits(x)


class DecoderStep(Graphed):
    def __init__(self, model: Decoder, R: int, dev, seed: int = 3):
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        self.model, self.R = model, R
        self.tokens = torch.randint(0, VOCAB, (R,), device=dev, generator=g)
        self.out = None

    def eager(self):
        self.out = self.model.forward(self.tokens)


class DecoderPart(Graphed):
    """One kernel class of a decoder step on static inputs: 'dense' (the 80 projections), 'moe' (40 x routing and
    experts) or 'head'."""

    def __init__(self, model: Decoder, part: str, R: int, dev):
        self.m, self.part = model, part
        self.h = rows_for(R, HIDDEN, dev, 31)
        self.core = rows_for(R, O_IN, dev, 32)
        self.y = torch.empty(R, sum(QKV_N), dtype=torch.bfloat16, device=dev)
        self.yo = torch.empty(R, HIDDEN, dtype=torch.bfloat16, device=dev)
        self.outs = (torch.empty(R, HIDDEN, dtype=torch.bfloat16, device=dev),
                     torch.empty(R, HIDDEN, dtype=torch.bfloat16, device=dev))
        self.logits = torch.empty(R, VOCAB, dtype=torch.bfloat16, device=dev)

    def eager(self):
        m = self.m
        if self.part == "dense":
            for blk in m.blocks:
                blk["qkv"].forward(self.h, out=self.y)
                blk["o"].forward(self.core, out=self.yo)
        elif self.part == "moe":
            for L, gate, _, _ in m.moe:
                m.G.route(self.h, gate, MOE_K, L, m.s)
                m.G.routed2(self.h, None, None, L, m.s, out=self.outs[0], out_shared=self.outs[1], k=MOE_K)
        else:
            m.head.forward(self.h, out=self.logits)


def decoder_bench(dev, steps: int, warmup: int, dist, peak: float) -> dict:
    model = Decoder(dev)
    res = {}
    for R in (1, 4, 8, 32):
        st = DecoderStep(model, R, dev)
        st.capture()
        ms = time_steps(st, steps, warmup, dist, dev)
        st.graph = None
        res[str(R)] = {"ms_per_step": ms, "tok_s": R / (ms * 1e-3)}
    # batch 1: the bytes a step reads (dense blocks, the experts each layer's routing picked, routers, head) and the
    # time by kernel class, each class replayed alone on static inputs; the rest is the torch stand-ins
    picks: list = []
    model.forward(DecoderStep(model, 1, dev).tokens, picks)
    torch.cuda.synchronize()
    moe_bytes = 0
    for p, (L, gate, ex, sh) in zip(picks, model.moe):
        for e in sorted(set(p[0].tolist())):
            moe_bytes += sum(mat_bytes(m) for m in (sh if e == L.shared_id else ex[e]))
        moe_bytes += gate.numel() * 2 + L.gate_w.numel() * 2
    step_bytes = model.layers * block_bytes() + moe_bytes + model.head_bytes()
    split = {}
    for part in ("dense", "moe", "head"):
        pt = DecoderPart(model, part, 1, dev)
        pt.capture()
        split[f"{part}_ms"] = time_steps(pt, steps, warmup, dist, dev)
        pt.graph = None
    product_ms = sum(split.values())
    split["torch_standins_ms"] = res["1"]["ms_per_step"] - product_ms
    split["product_ms"] = product_ms
    split["product_tok_s"] = 1.0 / (product_ms * 1e-3)      # this library's kernels alone, batch 1
    gbs = step_bytes / (res["1"]["ms_per_step"] * 1e-3) / 1e9
    return {"workload": "BASELINE configs[4]: 40-layer synthetic decoder (config-2 projections around stand-in mixer "
                        "cores, config-3 MoE in every layer, 6-bit mcg LM head to 248320, bf16 embedding), one decode "
                        "step, graph replay; batch 4 is the MTP-3 verification batch (3 drafted tokens + 1); mixer "
                        "cores, KV cache and the drafter are stand-ins outside this path",
            "batches": res, "mtp3_verify": {"rows": 4, **res["4"]},
            "roofline_batch1": {"bytes_per_step": step_bytes, "achieved_gbs": gbs, "peak": peak, "frac": gbs / peak,
                                "moe_mb_per_step": moe_bytes / 1e6, "head_mb": model.head_bytes() / 1e6},
            "split_batch1": split}


# ---------------------------------------------------------------------------------------------------------------
# the reference's own CUDA kernels (oracle/_ref), timed on the same workloads (reference arm only)
# ---------------------------------------------------------------------------------------------------------------
def ref_kernels(raw_blocks, dev, steps: int, warmup: int, moe_layers: int) -> dict:
    sys.path.insert(0, str(ROOT / "oracle"))
    import ref_host as RH
    if not RH.available():
        return {"unavailable": "oracle/_ref/espalier_ref_ext.so is not built (oracle/build_ref.py)"}
    out = {"what": "the reference's own kernels (its csrc/ built from its sources for sm_100a), driven with its own "
                   "host parameters (dense.plan, experts.tile_config, the fused-routing routed2 sequence), graph "
                   "replay on the same synthetic weights and rows as this library's arm"}
    blocks = [(RH.RefDense(qkv), RH.RefDense([o])) for qkv, o in raw_blocks]
    dense = {}
    for R in (1, 8, 32):
        st = Step(blocks, R, dev)
        st.eager()
        st.capture()
        ms = time_steps(st, steps, warmup, None, dev)
        st.graph = None
        dense[str(R)] = {"us_per_block": ms * 1e3 / len(blocks), "tok_s": R / (ms * 1e-3)}
    out["dense"] = dense
    del blocks
    raw = make_moe(moe_layers, dev)
    layers = [RH.RefMoE(r["ex"], r["sh"], r["gate_w"], r["gate"]) for r in raw]

    class _Ref(Graphed):
        def __init__(self, R):
            self.x = rows_for(R, MOE_D, dev, 21)
            self.o = [(torch.empty(R, MOE_D, dtype=torch.bfloat16, device=dev),
                       torch.empty(R, MOE_D, dtype=torch.bfloat16, device=dev)) for _ in layers]

        def eager(self):
            for L, (o, so) in zip(layers, self.o):
                L.forward(self.x, o, so)
    moe = {}
    for R in (1, 8, 32):
        st = _Ref(R)
        st.eager()
        st.capture()
        ms = time_steps(st, max(steps // 8, 10), warmup, None, dev)
        st.graph = None
        moe[str(R)] = {"us_per_layer": ms * 1e3 / len(layers)}
    out["moe"] = moe
    gate, sgate, copies = route_inputs(dev)
    rl = RH.RefMoE(raw[0]["ex"], raw[0]["sh"], sgate, gate)

    def call(x, g):
        rl.gate = g
        rl.route(x)

    def picks(R):
        return rl.pick[:R * rl.slots].view(R, rl.slots)[:, :MOE_K].cpu().numpy()
    out["route"] = route_bench(dev, max(steps // 8, 10), warmup, None, call, picks)["batches"]
    return out


def reference_arm(a, dev, metric: str, config: dict, ws: int):
    raw = make_blocks(a.layers, dev)
    runs = [cpu_baseline(raw, 1, a.layers, seconds=max(1.0, a.cpu_seconds / max(a.steps, 1) * 4))
            for _ in range(max(1, min(a.steps, 3)))]
    cb = runs[-1]
    line = {"metric": metric, "value": cb["value"], "unit": "tok/s", "n_gpus": ws, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": 1e3 / cb["value"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded random trellis codes)",
            "config": config, "impl": "reference", "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if not a.no_ref_kernels:
        line["ref_kernels"] = ref_kernels(raw, dev, max(a.steps, 10), a.warmup, a.moe_layers)
    return line


# ---------------------------------------------------------------------------------------------------------------
def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic_per_launch():
    """dram bytes of one config-2 block (qkv + o launches) from the committed ncu summary."""
    p = ROOT / "profiles" / "dense_traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text()).get("bytes_per_block")
        except (ValueError, KeyError):
            return None
    return None


def init_dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws <= 1:
        return None, 0, 1, 0
    import datetime

    import torch.distributed as dist
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    return dist, dist.get_rank(), ws, local


def probe(a, dev):
    """No timing: a few eager steps of one workload (for ncu captures)."""
    if a.probe == "dense":
        st = Step(our_blocks(make_blocks(2, dev)), a.probe_rows, dev)
    elif a.probe == "config1":
        from vllm_espalier_b200 import dense as D
        mats = config1_mats(dev)[:4]
        st = LayerStep([D.Dense([m]) for m in mats], rows_for(a.probe_rows, C1_K, dev, 7002), C1_N)
    elif a.probe == "route":
        call, _ = our_route(dev)
        gate, _, copies = route_inputs(dev)
        st = RouteStep(call, copies[:4], near_tie_rows(a.probe_rows, gate, MOE_K, dev, 4100 + a.probe_rows))
    else:
        from vllm_espalier_b200 import experts as G
        raw = make_moe(1, dev)
        st = MoEStep(G, [(G.prepare(r["ex"], r["sh"], r["gate_w"]), r["gate"]) for r in raw], a.probe_rows, dev)
    for _ in range(a.probe_iters):
        st.eager()
    torch.cuda.synchronize()
    print(json.dumps({"probe": a.probe, "rows": a.probe_rows, "iters": a.probe_iters}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--layers", type=int, default=40)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--moe-layers", type=int, default=32)
    ap.add_argument("--no-moe", action="store_true")
    ap.add_argument("--no-decoder", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the config1 and route blocks")
    ap.add_argument("--no-ref-kernels", action="store_true", help="reference arm: skip the reference's GPU kernels")
    ap.add_argument("--probe", choices=["dense", "moe", "config1", "route"], default=None,
                    help="no timing: run --probe-iters eager steps of one workload (for ncu captures)")
    ap.add_argument("--probe-rows", type=int, default=8)
    ap.add_argument("--probe-iters", type=int, default=3)
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)
    dist, rank, ws, local = init_dist()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if a.probe:
        probe(a, dev)
        return
    metric = "decode tok/s + compressed-weight HBM GB/s (% of peak) at batch 1/8/32, 1-8 GPU"
    config = {"workload": f"BASELINE configs[1]: fused dense decode of q/k/v/o blocks, hidden 2048, 4-bit int5, "
                          f"{a.layers} blocks a step (weights > L2, no flush)", "blocks": a.layers,
              "parallelism": f"dp{ws} replicas", "graph": not a.no_graph}

    if a.impl == "reference":
        if rank == 0:
            print(json.dumps(reference_arm(a, dev, metric, config, ws)))
        if dist:
            dist.destroy_process_group()
        return

    import vllm_espalier_b200 as pkg
    blocks = our_blocks(make_blocks(a.layers, dev))
    peak, peak_kind = peaks()
    gpu_index = local
    if os.environ.get("CUDA_VISIBLE_DEVICES"):
        gpu_index = int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local])
    clocks = Clocks(gpu_index)
    nbytes = block_bytes() * a.layers
    results, steps_main = {}, {}
    for R in (1, 8, 32):
        st = Step(blocks, R, dev)
        st.eager()
        if not a.no_graph:
            st.capture()
        steps_main[R] = st
        ms = time_steps(st, a.steps if R == 1 else max(a.steps // 4, 10), a.warmup, dist, dev)
        gbs = nbytes / (ms * 1e-3) / 1e9
        results[R] = {"tok_s": R * ws / (ms * 1e-3), "ms_per_step": ms, "weight_gbs": gbs, "hbm_frac": gbs / peak}
    clk = clocks.stop()
    e2e_ms, h2d, d2h = time_e2e(steps_main[1], a.steps, a.warmup, dist, dev)
    status = pkg._lib.device_status()
    r1 = results[1]
    line = {
        "metric": metric, "value": r1["tok_s"], "unit": "tok/s", "n_gpus": ws, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": r1["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp16", "dtype_note": "integer trellis decode to fp16 weights, fp16 x fp16 MMA with fp32 sums, bf16 in/out",
        "data": "synthetic (seeded random trellis codes, N(0,1) bf16 activations)", "config": config,
        "batches": {str(R): v for R, v in results.items()},
        "roofline": {"bound": "hbm", "achieved": r1["weight_gbs"], "peak": peak, "unit": "GB/s",
                     "frac": r1["weight_gbs"] / peak, "traffic": traffic_per_launch(),
                     "note": f"algorithmic compressed bytes {block_bytes()} a block / (step time / blocks) at batch 1; "
                             f"traffic = ncu dram bytes of one block's two launches; peak {peak_kind}"},
        "e2e": {"value": ws * 1 / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "gpu_launches": steps_main[1].launches() * a.steps,
        "clocks": clk, "device_status": status,
    }
    for st in steps_main.values():
        st.graph = None
    if rank == 0 and ws == 1 and not a.no_cpu:
        line["cpu_baseline"] = cpu_baseline(make_blocks(a.layers, dev), 1, a.layers, a.cpu_seconds)
    if not a.no_extra and ws == 1:
        line["config1"] = config1_bench(dev, max(a.steps // 8, 10), a.warmup, dist, peak,
                                        None if a.no_cpu else min(a.cpu_seconds, 5.0))
        call, picks = our_route(dev)
        line["route"] = route_bench(dev, max(a.steps // 8, 10), a.warmup, dist, call, picks)
    if not a.no_moe:
        line["moe"] = moe_bench(dev, a.moe_layers, max(a.steps // 16, 10), a.warmup, dist, peak, rank, ws)
        b8 = line["moe"]["batches"]["8"]
        line["ep_headline"] = {"metric": "MoE layer-stack decode tok/s at batch 8 a rank (config 3, expert parallel "
                                         "over the ranks)", "value": b8["tok_s_layer_stack"], "unit": "tok/s",
                               "scaling": "weak", "ep_bitwise": b8.get("ep_bitwise")}
    if not a.no_decoder and ws == 1:
        line["decoder"] = decoder_bench(dev, max(a.steps // 40, 5), a.warmup, dist, peak)
    line["device_status"] = pkg._lib.device_status()
    if rank == 0:
        print(json.dumps(line))
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
