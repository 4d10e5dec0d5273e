"""Routed and shared experts of one MoE layer for up to 32 tokens, every expert with its own width and codebook.

Surface kept from the reference (vllm_espalier/experts.py): prepare(experts, shared, gate_w) -> Layer,
scratch(layer, rows, slots, device) -> Scratch, route, routed2, windows, routed, dequant. The layer runs as

  route      (fused routing launch) router logits, softmax, top-k, renormalised weights, the shared expert as one more
             slot with its sigmoid gate, the grouping (distinct experts in id order, members in (row, slot) order) and,
             once the picks are out, H(x * suh) of every slot for gate and up, shared by all the launch's CTAs;
  rot_in     given vLLM's picks instead: group_shared does the shared slot and the grouping, rot_in the rotation
  moe_layer  one persistent launch: gate and up of every distinct expert (weights decoded in registers, K in S
             slices), the SwiGLU epilogue, down, and each row's slot-ordered weighted sum written in x's dtype
             (ESPALIER_MOE_FUSED=0: the same work as two launches, moe_gateup then moe_down, same bits)

Every sum has a fixed order that depends on the shapes only, so a token's output never depends on the other tokens,
and nothing allocates during a forward, so CUDA graphs capture it. Trellises are read in place through pointer tables;
each projection's suh / svh are stacked once and the matrices keep views of their rows.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from . import codebooks
from ._env import MOE_ONE_LAUNCH
from ._lib import ext, lib
from .matrix import dequant  # noqa: F401  (part of this module's reference surface)

KERNEL_CB = codebooks.KERNEL_CB
COMPILED = codebooks.COMPILED
PROJECTIONS = ("gate", "up", "down")
ACT_F32 = 1                      # gateup_epilogue's activation mode: SwiGLU in fp32


def gateup_splits(D: int, I: int, slots: int) -> int:
    """K slices S of the gate/up work: enough (expert, column block, slice) items to give every SM one for a single
    token's slots, each slice at least 8 k-tiles. A function of the shapes (and top-k) only."""
    sms = max(1, lib().esp_sm_count())
    s = max(1, sms // max(1, slots * (I // 128)))
    while s > 1 and D // 16 < 8 * s:
        s -= 1
    return s


@dataclass
class Projection:
    """One projection of every table entry: what the grouped kernels read."""

    ptr: torch.Tensor        # int64 [E] trellis addresses (device)
    k2: torch.Tensor         # int32 [E] half-bits a weight (device)
    cb: torch.Tensor         # int32 [E] kernel codebook ids (device)
    k2_host: torch.Tensor    # CPU copies, for the host-side check of the (codebook, width) pairs
    cb_host: torch.Tensor
    suh: torch.Tensor        # fp16 [E, in]
    svh: torch.Tensor        # fp16 [E, out]


@dataclass
class Layer:
    gate: Projection
    up: Projection
    down: Projection
    E: int                   # table entries: the routed experts, then the shared expert if there is one
    D: int                   # hidden size
    I: int                   # intermediate size
    shared_id: int = -1      # the shared expert's entry (E - 1), -1 without one
    gate_w: torch.Tensor | None = None       # the shared expert's sigmoid-gate weight [D], the model's dtype
    keep: list = field(default_factory=list, repr=False)   # the trellises the pointer tables point into
    _host: dict = field(default_factory=dict, repr=False)

    def projection(self, j: int) -> Projection:
        return (self.gate, self.up, self.down)[j]

    def host_tables(self, which: str) -> tuple[torch.Tensor, torch.Tensor]:
        """CPU int32 (k2, cb) tables of 'gu' ([2][E]: gate, up), 'd' ([E]) or 'all' ([3][E]); built once, kept alive
        (the C calls read them)."""
        if which not in self._host:
            ps = {"gu": (self.gate, self.up), "d": (self.down,), "all": (self.gate, self.up, self.down)}[which]
            self._host[which] = (torch.cat([p.k2_host for p in ps]).contiguous(),
                                 torch.cat([p.cb_host for p in ps]).contiguous())
        return self._host[which]


def _projection(entries, j: int, kin: int, n: int, dev) -> Projection:
    E = len(entries)
    suh = torch.empty((E, kin), dtype=torch.float16, device=dev)
    svh = torch.empty((E, n), dtype=torch.float16, device=dev)
    ptr, k2, cb = [], [], []
    for e, mats in enumerate(entries):
        m = mats[j]
        what = f"expert {e} {PROJECTIONS[j]}"
        if (m.in_features, m.out_features) != (kin, n):
            raise ValueError(f"{what}: {m.in_features}x{m.out_features}, the layer wants {kin}x{n}")
        if m.trellis.dtype != torch.int16 or not m.trellis.is_contiguous() or m.trellis.device != dev:
            raise ValueError(f"{what}: trellis must be contiguous int16 on {dev}")
        cb.append(codebooks.kernel_id(m.cb, m.K, what))
        k2.append(2 * m.K)
        ptr.append(m.trellis.data_ptr())
        suh[e].copy_(m.suh.reshape(-1))
        svh[e].copy_(m.svh.reshape(-1))
        m.suh, m.svh = suh[e], svh[e]       # the matrix now reads its row of the stacks
    host = torch.tensor([k2, cb], dtype=torch.int32)
    return Projection(torch.tensor(ptr, dtype=torch.int64, device=dev), host[0].to(dev), host[1].to(dev),
                      host[0].clone(), host[1].clone(), suh, svh)


def prepare(experts, shared=None, gate_w=None) -> Layer:
    """experts: [(gate, up, down)] coded matrices in expert-id order; shared: the shared expert's (gate, up, down),
    appended as the last entry, with gate_w the weight [D] of its sigmoid gate."""
    entries = list(experts) + ([tuple(shared)] if shared is not None else [])
    if not entries:
        raise ValueError("an MoE layer needs at least one expert")
    D, I = entries[0][0].in_features, entries[0][0].out_features
    dev = entries[0][0].trellis.device
    gate, up, down = (_projection(entries, j, kin, n, dev) for j, (kin, n) in enumerate(((D, I), (D, I), (I, D))))
    return Layer(gate, up, down, len(entries), D, I, len(entries) - 1 if shared is not None else -1,
                 None if gate_w is None else gate_w.reshape(-1).contiguous(),
                 [m.trellis for mats in entries for m in mats])


class Scratch:
    """Device buffers for `rows` tokens of `slots` picks (the shared slot included), shared by every layer of one shape
    (layers run one after another on a stream). Counters are zero on entry and left zero by every launch."""

    def __init__(self, E: int, D: int, I: int, rows: int, slots: int, device):
        P, maxu = rows * slots, min(rows * slots, E)
        self.rows, self.slots, self.E, self.P, self.maxu = rows, slots, E, P, maxu
        self.S = gateup_splits(D, I, slots)
        spec = {   # name: (elements, dtype, initial value)
            "xg": (P * D, torch.float16, 0), "xu": (P * D, torch.float16, 0), "xd": (P * I, torch.float16, 0),
            "z": (P * max(2 * self.S * I, D), torch.float32, 0), "y": (P * D, torch.float32, 0),
            "logits": (rows * (E + 1), torch.float32, 0), "route_counter": (3, torch.int32, 0),
            "pick": (P, torch.int32, 0), "wts": (P, torch.float32, 0), "ids": (maxu, torch.int32, 0),
            "count": (1, torch.int32, 0), "members": (maxu * rows, torch.int32, -1),
            "cnt_gu": (maxu * (I // 128) + 1, torch.int32, 0), "cnt_d": (rows * (D // 128) + 1, torch.int32, 0),
            "cnt_layer": (int(lib().esp_moe_layer_counters(maxu, rows, D, I)), torch.int32, 0),
        }
        for name, (n, dtype, v) in spec.items():
            setattr(self, name, torch.full((max(n, 1),), v, dtype=dtype, device=device))
        self.xg, self.xu, self.y = self.xg.view(P, D), self.xu.view(P, D), self.y.view(P, D)
        self.xd = self.xd.view(P, I)
        self.rotated = False    # route() also wrote xg / xu for its rows (the routing launch did rot_in's work)

    def window(self, R: int):
        """(ids, members [maxu, R]) of a call with R rows: the grouping's layout depends on R."""
        maxu = min(R * self.slots, self.E)
        return self.ids[:maxu], self.members[:maxu * R].view(maxu, R)


_SCRATCH: dict[tuple, Scratch] = {}


def scratch(layer: Layer, rows: int, slots: int, device) -> Scratch:
    """The shared Scratch of the layer's shape (slots counts the shared slot when the layer has one)."""
    key = (layer.E, layer.D, layer.I, rows, slots, str(torch.device(device)))
    if key not in _SCRATCH:
        _SCRATCH[key] = Scratch(layer.E, layer.D, layer.I, rows, slots, device)
    return _SCRATCH[key]


def _fits(R: int, slots: int, s: Scratch):
    if R > s.rows or slots != s.slots:
        raise ValueError(f"{R} rows of {slots} slots, but the scratch holds {s.rows} rows of {s.slots}")


def route(x: torch.Tensor, gate: torch.Tensor, k: int, L: Layer, s: Scratch):
    """Fused routing of x [R, D] with router weight gate [E_routed, D] into the scratch (pick, wts, ids, count,
    members), the shared expert as slot k when the layer has one, and in the same launch the experts' input rotation
    (rot_in's xg / xu); routed2(x, pick=None) then runs the experts on the same x."""
    R = x.shape[0]
    _fits(R, k + (L.shared_id >= 0), s)
    ids, members = s.window(R)
    n = R * s.slots
    e = ext()
    e.route_group(x, gate, L.gate_w, k, L.shared_id, s.logits, s.route_counter, s.pick[:n], s.wts[:n], ids, s.count,
                  members, rotate=(L.gate.suh, L.up.suh, s.xg, s.xu, L.E))
    s.rotated = True


def routed2(x: torch.Tensor, pick: torch.Tensor | None, wts: torch.Tensor | None, L: Layer, s: Scratch,
            out: torch.Tensor | None = None, out_shared: torch.Tensor | None = None, k: int | None = None):
    """x [R, D] in the model's dtype; pick int32 [R, k] (vLLM's routed ids; outside [0, E) skipped) and wts fp32
    [R, k], or pick=None after route() (then k is given). Returns (routed sum, gated shared output or None), [R, D]
    in x's dtype."""
    e = ext()
    R = x.shape[0]
    if pick is not None:
        k = pick.shape[1]
    has_shared = L.shared_id >= 0
    slots = k + has_shared
    _fits(R, slots, s)
    ids, members = s.window(R)
    P = R * slots
    pk, wt = s.pick[:P], s.wts[:P]
    if pick is not None:
        e.group_shared(pick, wts, x, x.stride(0), L.gate_w, L.shared_id, pk, wt, ids, s.count, members, R, k, L.E)
    if pick is not None or not s.rotated:
        e.rot_in(x, x.stride(0), pk, L.gate.suh, L.up.suh, s.xg, s.xu, R, L.D, slots, L.E)
    s.rotated = False
    out = out if out is not None else torch.empty((R, L.D), dtype=x.dtype, device=x.device)
    if has_shared and out_shared is None:
        out_shared = torch.empty((R, L.D), dtype=x.dtype, device=x.device)
    sh = out_shared if has_shared else None
    if MOE_ONE_LAUNCH:
        e.moe_layer(s.xg, s.xu, L, ids, s.count, members, pk, wt, slots, k, R, s.S, s.z, s.xd, s.y, s.cnt_layer,
                    out, sh)
    else:
        e.moe_gateup(s.xg, s.xu, L, ids, s.count, members, slots, P, s.S, s.z, s.cnt_gu, s.xd)
        e.moe_down(s.xd, L, ids, s.count, members, pk, wt, slots, k, R, s.y, s.cnt_d, out, sh)
    return out, sh


def windows(x: torch.Tensor, pick: torch.Tensor | None, wts: torch.Tensor | None, L: Layer, s: Scratch,
            k: int | None = None, gate: torch.Tensor | None = None):
    """routed2 over consecutive windows of s.rows tokens (prefill), each window exactly as in decode; with gate (and
    pick=None) each window is routed first. Returns (routed sum, shared output or None)."""
    out = torch.empty_like(x)
    sh = torch.empty_like(x) if L.shared_id >= 0 else None
    for lo in range(0, x.shape[0], s.rows):
        rows = slice(lo, lo + s.rows)
        if gate is not None:
            route(x[rows], gate, k, L, s)
        routed2(x[rows], None if pick is None else pick[rows], None if wts is None else wts[rows], L, s,
                out=out[rows], out_shared=None if sh is None else sh[rows], k=k)
    return out, sh


def routed(x: torch.Tensor, pick: torch.Tensor, wts: torch.Tensor, L: Layer, s: Scratch,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """The weighted sum of the picked experts, fp32 [R, D], through the reference's separate kernels: group, rot_in,
    grouped (gate and up, K in s.S slices), gateup_epilogue, grouped (down), down_combine. Picks outside [0, E) are
    skipped; every slot is a routed slot."""
    e = ext()
    R, slots = pick.shape
    _fits(R, slots, s)
    ids, members = s.window(R)
    D, I, E, P, S = L.D, L.I, L.E, R * slots, s.S
    e.group(pick, ids, s.count, members, R, slots, E)
    e.rot_in(x, x.stride(0), pick, L.gate.suh, L.up.suh, s.xg, s.xu, R, D, slots, E)
    e.grouped(s.xg, s.xu, L.gate.ptr, L.up.ptr, L.gate.k2, L.up.k2, L.gate.cb, L.up.cb, ids, s.count, members, s.z,
              2, D, I, P, S, slots, tables=L.host_tables("gu"))
    e.gateup_epilogue(s.z, pick, L.gate.svh, L.up.svh, L.down.suh, s.xd, R, P, I, S, slots, E, math.inf, ACT_F32)
    e.grouped(s.xd, s.xd, L.down.ptr, L.down.ptr, L.down.k2, L.down.k2, L.down.cb, L.down.cb, ids, s.count, members,
              s.z, 1, I, D, P, 1, slots, tables=L.host_tables("d"))
    out = out if out is not None else torch.empty((R, D), dtype=torch.float32, device=x.device)
    e.down_combine(s.z, pick, L.down.svh, s.y, wts, out, R, P, D, 1, slots, E)
    return out
