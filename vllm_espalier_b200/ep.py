"""Expert-parallel MoE layer over the ranks of one box (one process a GPU, torch.distributed over NCCL).

The reference runs a MoE layer on one GPU (vllm_espalier/experts.py routed2); this is the sharded form of the same
layer, with outputs bit-identical to it for every world size:

  * rank q holds routed experts [q E / world, (q + 1) E / world) (contiguous blocks: 128 / 64 / 32 at 2 / 4 / 8 ranks)
    plus the shared expert; the router and the shared gate are replicated.
  * each rank routes its own rows with the fused routing kernel (the same bits as on one GPU);
  * dispatch: every row and its pick list go to every rank in one all_to_all ([world][R][2 D + 4 slots] bytes: the
    bf16 row, then its int32 picks; fixed sizes, so the step is CUDA-graph capturable and the exchange is at most
    8 x 32 x 4 KiB = 1 MiB a rank);
  * each rank maps the received picks to its local expert ids (the shared slot is local only on the row's home rank),
    groups them (an expert with more than 32 members takes several entries) and runs rot_in, the fused gate/up and
    the fused down kernels on all received rows, producing fp32 y rows per slot;
  * combine: the y rows go back to their home rank (one all_to_all of [world][R][slots][D] fp32), which sums each
    row's routed slots in slot order with fp32 fused multiply-adds from 0 (esp_ep_combine): the single-GPU kernel's
    arithmetic on the same y values, hence the same output bits.

The exchange (ESPALIER_EP_EXCHANGE): `p2p` (default) moves rows and results by stores into the other ranks' memory
(csrc/ep.cu, PeerExchange below): a row goes only to the ranks owning one of its picks, a slot's y row only from its
owner to its home rank, with release / acquire flags instead of collectives; a layer is four launches (routing,
esp_ep_in = dispatch + receive + grouping + rotation, the one-launch expert kernel storing each slot's y row in its
home rank's inbox, esp_ep_out = the combine) and nothing on the host; `nccl` is the two-collective form above. The index logic of the `nccl` form (local
tables, owners, buffer layouts) is in plain torch functions shared with the CPU tests (gloo ranks with a stand-in
expert function); the `p2p` form computes the same table on the device (esp_ep_in).
"""
from __future__ import annotations

import ctypes as C

import torch

from ._env import EP_EXCHANGE
from ._lib import DTYPE, check, ext, lib, stream_ptr
from . import experts as X

MAXM = 32   # members an entry of the receiver's grouping


def expert_range(rank: int, world: int, E: int) -> tuple[int, int]:
    """Routed experts [e0, e1) held by `rank`."""
    return rank * E // world, (rank + 1) * E // world


def owner_of(e: torch.Tensor, world: int, E: int) -> torch.Tensor:
    """Rank holding routed expert e (the largest q with q E / world <= e)."""
    return ((e + 1) * world - 1) // E


def local_table(recv_pick: torch.Tensor, rank: int, world: int, E: int, n_routed: int) -> torch.Tensor:
    """recv_pick int32 [world][R][slots] (global ids, the shared slot = slot n_routed with id E) -> the receiving rank's
    pick table: local routed ids e - e0 for its experts, nl (the local shared entry) for the shared slot of its own rows
    only, -1 elsewhere."""
    e0, e1 = expert_range(rank, world, E)
    nl = e1 - e0
    lp = torch.where((recv_pick >= e0) & (recv_pick < e1), recv_pick - e0, torch.full_like(recv_pick, -1))
    if recv_pick.shape[2] > n_routed:
        src = torch.arange(world, device=recv_pick.device).view(world, 1)
        sh = recv_pick[:, :, n_routed]
        lp[:, :, n_routed] = torch.where((src == rank) & (sh >= 0), torch.full_like(sh, nl), torch.full_like(sh, -1))
    return lp


def dispatch(x: torch.Tensor, pick: torch.Tensor, world: int, group=None):
    """Every row and its pick list to every rank, in one collective: a row travels as the bytes of its D values
    followed by those of its int32 picks. Returns (recv_x [world][R][D] (a strided view), recv_pick
    [world][R][slots])."""
    import torch.distributed as dist
    R, D = x.shape
    slots = pick.shape[1]
    nb = x.element_size() * D
    row = torch.cat([x.contiguous().view(torch.uint8).view(R, nb), pick.contiguous().view(torch.uint8).view(R, 4 * slots)],
                    1)                                         # bytes: neither NCCL nor gloo has a 16-bit integer type
    send = row.unsqueeze(0).expand(world, R, nb + 4 * slots).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv[:, :, :nb].view(x.dtype), recv[:, :, nb:].contiguous().view(torch.int32)


def give_back(y: torch.Tensor, group=None) -> torch.Tensor:
    """y fp32 [world][R][slots][D] (rows received from each source) -> the same layout indexed by owner on the home
    rank."""
    import torch.distributed as dist
    out = torch.empty_like(y)
    dist.all_to_all_single(out, y.contiguous(), group=group)
    return out


def _device_view(ptr: int, n: int, dtype: torch.dtype, device) -> torch.Tensor:
    """A torch tensor over n elements of raw device memory (no copy), through the CUDA array interface."""
    typestr = {torch.int32: "<i4", torch.float32: "<f4", torch.int16: "<i2"}[torch.int16 if dtype.itemsize == 2 else dtype]

    class _Raw:
        __cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}
    t = torch.as_tensor(_Raw(), device=device)
    return t.view(dtype) if dtype.itemsize == 2 else t


class PeerExchange:
    """This rank's inboxes (one allocation, shared with every other rank through a CUDA IPC handle) and the mapped
    inboxes of the others, for rows of up to `rows` tokens a rank: x [world][rows][D], picks [world][rows][slots],
    y fp32 [rows][slots][D], flags_x / flags_y [world], the epoch, counters. Built once per layer at set-up."""

    LAYOUT = ("x", "pick", "y", "flags_x", "flags_y", "epoch", "done", "count")

    def __init__(self, rank: int, world: int, rows: int, D: int, slots: int, dtype: torch.dtype, device, group=None):
        import torch.distributed as dist
        h = lib()
        sizes = {"x": world * rows * D * dtype.itemsize, "pick": world * rows * slots * 4, "y": rows * slots * D * 4,
                 "flags_x": world * 4, "flags_y": world * 4, "epoch": 4, "done": world * 4, "count": 4}
        self.offset, total = {}, 0
        for name in self.LAYOUT:
            self.offset[name] = total
            total += -(-sizes[name] // 256) * 256
        base, handle = C.c_void_p(), (C.c_char * int(h.esp_ipc_handle_bytes()))()
        check(h.esp_ipc_alloc(total, C.byref(base), handle))
        self.base, self.rank, self.world = base.value, rank, world
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.bases, self.opened = [], []
        for q in range(world):
            if q == rank:
                self.bases.append(self.base)
                continue
            p = C.c_void_p()
            check(h.esp_ipc_open(C.create_string_buffer(handles[q], len(handles[q])), C.byref(p)))
            self.bases.append(p.value)
            self.opened.append(p.value)
        self.peer = {name: (C.c_void_p * world)(*[b + self.offset[name] for b in self.bases])
                     for name in ("x", "pick", "y", "flags_x", "flags_y")}
        self.inbox_x = _device_view(self.local("x"), world * rows * D, dtype, device).view(world * rows, D)
        self.lp = torch.full((world * rows * slots,), -1, dtype=torch.int32, device=device)

    def local(self, name: str) -> int:
        return self.base + self.offset[name]

    def close(self):
        h = lib()
        for p in self.opened:
            h.esp_ipc_close(C.c_void_p(p))
        self.opened = []
        if self.base:
            h.esp_ipc_free(C.c_void_p(self.base))
            self.base = 0


class EPLayer:
    """One MoE layer's local share on this rank. `local_experts`: the (gate, up, down) matrices of experts
    [e0, e1) = expert_range(rank, world, E); `shared`: the shared expert's, `gate_w` its sigmoid-gate weight."""

    def __init__(self, local_experts, shared, gate_w: torch.Tensor, rank: int, world: int, E: int, rows: int = 32,
                 k: int = 8):
        e0, e1 = expert_range(rank, world, E)
        if len(local_experts) != e1 - e0:
            raise ValueError(f"rank {rank} of {world} holds experts [{e0}, {e1}), got {len(local_experts)}")
        self.rank, self.world, self.E, self.k = rank, world, E, k
        self.L = X.prepare(local_experts, shared, gate_w)          # local ids 0..nl-1, the shared entry nl
        self.nl = e1 - e0
        self.gate_w = self.L.gate_w
        dev = gate_w.device
        D, I = self.L.D, self.L.I
        self.slots = k + 1
        self.rows = rows
        # the home side: routing of this rank's rows (global ids, shared id = E)
        self.rs = X.Scratch(E, D, I, rows, self.slots, dev)
        # the expert side: all ranks' rows
        P = world * rows * self.slots
        self.P = P
        self.maxu = min(P, self.nl + 1 + P // MAXM + 1)
        self.S = X.gateup_splits(D, I, self.slots)
        self.xg = torch.zeros((P, D), dtype=torch.float16, device=dev)
        self.xu = torch.zeros((P, D), dtype=torch.float16, device=dev)
        self.xd = torch.zeros((P, I), dtype=torch.float16, device=dev)
        self.z = torch.zeros((P * max(2 * self.S * I, D),), dtype=torch.float32, device=dev)
        self.y = torch.zeros((P, D), dtype=torch.float32, device=dev)
        self.ids = torch.zeros((self.maxu,), dtype=torch.int32, device=dev)
        self.count = torch.zeros((1,), dtype=torch.int32, device=dev)
        self.members = torch.full((self.maxu, MAXM), -1, dtype=torch.int32, device=dev)
        self.cnt_gu = torch.zeros((self.maxu * (I // 128) + 1,), dtype=torch.int32, device=dev)
        self.cnt_d = torch.zeros((world * rows * (D // 128) + 1,), dtype=torch.int32, device=dev)
        self.cnt_layer = torch.zeros((int(lib().esp_moe_layer_counters(self.maxu, world * rows, D, I)),),
                                     dtype=torch.int32, device=dev)
        self.no_w = torch.zeros((P,), dtype=torch.float32, device=dev)
        self.no_out = torch.empty((world * rows, D), dtype=torch.bfloat16, device=dev)
        self.exchange = EP_EXCHANGE
        self.ex = None          # the PeerExchange, made at the first p2p forward (it needs the rows' dtype)

    def route(self, x: torch.Tensor, gate: torch.Tensor):
        """Fused routing of this rank's rows -> (pick int32 [R][slots], wts fp32 [R][slots]), global ids."""
        R = x.shape[0]
        s = self.rs
        ids, members = s.window(R)
        ext().route_group(x, gate, self.gate_w, self.k, self.E, s.logits, s.route_counter, s.pick[:R * self.slots],
                          s.wts[:R * self.slots], ids, s.count, members)
        return s.pick[:R * self.slots].view(R, self.slots), s.wts[:R * self.slots].view(R, self.slots)

    def experts(self, recv_x: torch.Tensor, lp: torch.Tensor) -> torch.Tensor:
        """y fp32 [world][R][slots][D] of the local experts for every received (row, slot) with a local pick; recv_x
        [world][R][D] (any row stride)."""
        world, R, D = recv_x.shape
        if R > self.rows:
            raise ValueError(f"{R} rows a rank, the layer holds {self.rows}")
        self._run_experts(recv_x, recv_x.stride(1), world * R, lp.reshape(-1))
        return self.y[:world * R * self.slots].view(world, R, self.slots, D)

    def _run_experts(self, rows_x, stride: int, rows: int, lpf: torch.Tensor):
        e, L, D, slots = ext(), self.L, self.L.D, self.slots
        e.group(lpf, self.ids, self.count, self.members, rows, slots, self.nl + 1)
        e.rot_in(rows_x, stride, lpf, L.gate.suh, L.up.suh, self.xg, self.xu, rows, D, slots, self.nl + 1)
        self._expert_kernels(rows, lpf)

    def _expert_kernels(self, rows: int, lpf: torch.Tensor):
        """The y rows of every slot with a local pick (xg / xu rotated, the grouping in ids / count / members); no
        combine here (n_routed 0: the home rank combines). The one-launch kernel holds up to 32 rows; above (world x R
        received rows) the two launches run."""
        e, L, slots = ext(), self.L, self.slots
        if X.MOE_ONE_LAUNCH and rows <= 32:
            e.moe_layer(self.xg, self.xu, L, self.ids, self.count, self.members, lpf, self.no_w, slots, 0, rows, self.S,
                        self.z, self.xd, self.y, self.cnt_layer, self.no_out[:rows], None)
        else:
            e.moe_gateup(self.xg, self.xu, L, self.ids, self.count, self.members, slots, rows * slots, self.S, self.z,
                         self.cnt_gu, self.xd)
            e.moe_down(self.xd, L, self.ids, self.count, self.members, lpf, self.no_w, slots, 0, rows, self.y,
                       self.cnt_d, self.no_out[:rows], None)

    def forward(self, x: torch.Tensor, gate: torch.Tensor, out: torch.Tensor | None = None,
                out_shared: torch.Tensor | None = None, group=None):
        """x [R, D] bf16/fp16 (this rank's rows), gate [E, D] the router -> (routed sum, shared output), [R, D] in x's
        dtype, bit-identical to experts.routed2 on one GPU holding every expert."""
        R, D = x.shape
        if self.exchange == "p2p":
            return self._forward_p2p(x, gate, out, out_shared, group)
        pick, wts = self.route(x, gate)
        recv_x, recv_p = dispatch(x, pick, self.world, group)
        lp = local_table(recv_p, self.rank, self.world, self.E, self.k)
        y = self.experts(recv_x, lp)
        back = give_back(y, group)
        out = out if out is not None else torch.empty((R, D), dtype=x.dtype, device=x.device)
        out_shared = out_shared if out_shared is not None else torch.empty((R, D), dtype=x.dtype, device=x.device)
        check(lib().esp_ep_combine(back.data_ptr(), pick.data_ptr(), wts.data_ptr(), out.data_ptr(),
                                   out_shared.data_ptr(), DTYPE[out.dtype], R, D, self.slots, self.k, self.E,
                                   self.world, self.rank, stream_ptr(x.device)))
        return out, out_shared

    def _forward_p2p(self, x, gate, out, out_shared, group):
        """The same layer with the peer-store exchange, four launches: routing; esp_ep_in (dispatch, receive, grouping,
        the experts' input rotation); the expert layer kernel, storing each slot's y row in its home rank's inbox (up to
        32 received rows; above, the two expert launches and esp_ep_out's return step); esp_ep_out (the combine)."""
        R, D = x.shape
        if R > self.rows:
            raise ValueError(f"{R} rows a rank, the layer holds {self.rows}")
        if self.ex is None:
            self.ex = PeerExchange(self.rank, self.world, self.rows, D, self.slots, x.dtype, x.device, group)
        ex, h, st = self.ex, lib(), stream_ptr(x.device)
        world, rank, slots, k = self.world, self.rank, self.slots, self.k
        pick, wts = self.route(x, gate)
        x = x if x.stride(1) == 1 else x.contiguous()
        L, lp = self.L, ex.lp[:world * R * slots]
        check(h.esp_ep_in(x.data_ptr(), DTYPE[x.dtype], x.stride(0), R, D, pick.data_ptr(), slots, k, self.E, world,
                          rank, ex.peer["x"], ex.peer["pick"], ex.peer["flags_x"], ex.local("epoch"), lp.data_ptr(),
                          self.ids.data_ptr(), self.count.data_ptr(), self.members.data_ptr(), MAXM, self.maxu,
                          L.gate.suh.data_ptr(), L.up.suh.data_ptr(), self.xg.data_ptr(), self.xu.data_ptr(), st))
        rows = world * R
        returned = X.MOE_ONE_LAUNCH and rows <= 32
        if returned:    # the expert kernel stores each slot's y row in its home rank's inbox and releases the flags
            ext().moe_layer_ep(self.xg, self.xu, L, self.ids, self.count, self.members, lp, self.no_w, slots, rows,
                               self.S, self.z, self.xd, self.cnt_layer, ex.peer["y"], ex.peer["flags_y"],
                               ex.local("epoch"), world, rank, R, self.y)
        else:
            self._expert_kernels(rows, lp)
        out = out if out is not None else torch.empty((R, D), dtype=x.dtype, device=x.device)
        out_shared = out_shared if out_shared is not None else torch.empty((R, D), dtype=x.dtype, device=x.device)
        check(h.esp_ep_out(self.y.data_ptr(), lp.data_ptr(), world, rank, R, slots, k, self.E, D, ex.peer["y"],
                           ex.peer["flags_y"], pick.data_ptr(), wts.data_ptr(), out.data_ptr(), out_shared.data_ptr(),
                           DTYPE[out.dtype], ex.local("epoch"), ex.local("done"), ex.local("count"), int(returned), st))
        return out, out_shared
