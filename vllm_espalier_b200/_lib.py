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
    "esp_route_group": (I, [P, I, L, I, I, P, I, P, I, I, P, P, P, P, P, P, P, I, I, P]),
    "esp_group": (I, [P, I, I, I, P, P, P, I, I, P]),
    "esp_group_shared": (I, [P, P, P, I, L, I, P, I, P, P, P, P, P, I, I, I, I, I, P]),
    "esp_rot_in": (I, [P, I, L, P, P, P, P, P, I, I, I, I, P]),
    "esp_grouped": (I, [P, P, P, P, P, P, P, P, P, P, I, P, P, P, I, I, P, I, I, I, I, I, I, P]),
    "esp_moe_gateup": (I, [P, P, P, P, P, P, P, P, P, P, I, P, P, P, P, P, P, I, I, I, I, I, I, I, P, P, P, P]),
    "esp_moe_down": (I, [P, P, P, P, P, P, I, P, P, P, P, I, I, P, P, I, I, I, I, I, P, P, P, P, I, P]),
    "esp_gateup_epilogue": (I, [P, P, P, P, P, P, I, I, I, I, I, I, F, I, P]),
    "esp_down_combine": (I, [P, P, P, P, P, P, P, I, I, I, I, I, I, I, I, I, P]),
    "esp_combine": (I, [P, P, P, I, I, I, P]),
    "esp_ep_combine": (I, [P, P, P, P, P, I, I, I, I, I, I, I, I, P]),
    "esp_wait_flag": (I, [P, I, P, P]),
    "esp_moe_layer": (I, [P, P, P, P, P, P, P, P, P, P, P, P, P, I, P, P, P, P, P, P, P, I, I, P, P, I, I, I, I, I, I,
                          P, P, P, P, P, P, I, P]),
    "esp_moe_layer_counters": (S, [I, I, I, I]),
    "esp_dense_z_bytes": (S, [I]),
    "esp_route_rot": (I, [P, I, L, I, I, P, I, P, I, I, P, P, P, P, P, P, P, I, I, P, P, P, P, I, P]),
    "esp_ipc_handle_bytes": (S, []),
    "esp_ipc_alloc": (I, [S, C.POINTER(P), P]),
    "esp_ipc_open": (I, [P, C.POINTER(P)]),
    "esp_ipc_close": (I, [P]),
    "esp_ipc_free": (I, [P]),
    "esp_ep_in": (I, [P, I, L, I, I, P, I, I, I, I, I, C.POINTER(P), C.POINTER(P), C.POINTER(P), P, P, P, P, P, I, I,
                      P, P, P, P, P]),
    "esp_moe_layer_ep": (I, [P, P, P, P, P, P, P, P, P, P, P, P, P, I, P, P, P, P, P, P, P, I, I, P, P, I, I, I, I, I,
                             P, P, P, C.POINTER(P), C.POINTER(P), P, I, I, I, P, P]),
    "esp_ep_out": (I, [P, P, I, I, I, I, I, I, I, C.POINTER(P), C.POINTER(P), P, P, P, P, I, P, P, P, I, P]),
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


_private_z: dict = {}


def _z_for(Z: torch.Tensor, M: int, device) -> torch.Tensor:
    """The split-K scratch for ext().dense: a private per-device buffer, zeroed when it is made and left zero by every
    call (the kernel's tagged partials need a zero Z on entry), sized for 32 rows. The caller's Z is accepted and not
    used: the reference allocates it with torch.empty (vllm_espalier/dense.py:42-48), and sizes it by its own plan.
    Only the Python shim allocates; the C ABI never does."""
    need = int(lib().esp_dense_z_bytes(max(M, 32)))
    z = _private_z.get(device)
    if z is None or z.numel() * 4 < need:
        z = torch.zeros(need // 4, dtype=torch.float32, device=device)
        _private_z[device] = z
    return z


class _Ext:
    """The reference extension's functions over the C ABI."""

    # ---- dense layer (experts.cpp:193-211) ----
    @staticmethod
    def dense(x, T, suh, svh, col0, y, xh, Z, counters, k2, cb, SK=1, W=4, PF=1, rot_smem=0):
        """SK / W / PF / rot_smem are the reference's tile-plan hints; this library plans its own split (k-slices of
        every 128-column block over all SMs) from the shape alone, so they are accepted and ignored."""
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
        Z = _z_for(Z, M, x.device)
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


    # ---- MoE (experts.cpp:44-190, 214-223) ----
    @staticmethod
    def route_group(x, gate, sgate, k, shared_id, logits, counter, pick_out, wts_out, uids, ucount, members,
                    rotate=None):
        """rotate = (suh_g, suh_u, xg, xu, E_tables): this library's fused form, which also writes rot_in's output
        (counter: 3 int32 words)."""
        _need(x.is_cuda and x.dim() == 2 and x.stride(1) == 1 and gate.is_contiguous(), "x / gate layout")
        _need(gate.dtype == x.dtype and x.dtype in (torch.bfloat16, torch.float16), "gate and x must share a dtype")
        _check(logits, torch.float32, "logits")
        _check(counter, torch.int32, "counter")
        R, H = x.shape
        E = gate.shape[0]
        has = shared_id >= 0
        _need(logits.numel() >= R * (E + has), "logits scratch too small")
        maxm = members.size(1) if members.dim() == 2 else R
        args = (x.data_ptr(), DTYPE[x.dtype], x.stride(0), R, H, gate.data_ptr(), E, ptr(sgate), int(k),
                int(shared_id), logits.data_ptr(), counter.data_ptr(), pick_out.data_ptr(), wts_out.data_ptr(),
                uids.data_ptr(), ucount.data_ptr(), members.data_ptr(), maxm, uids.numel())
        if rotate is None:
            check(lib().esp_route_group(*args, stream_ptr(x.device)))
            return
        suh0, suh1, out0, out1, e_tab = rotate
        _need(counter.numel() >= 3, "counter: 3 int32 words for the fused rotation")
        for t, n in ((suh0, "suh_g"), (suh1, "suh_u"), (out0, "xg"), (out1, "xu")):
            _check(t, torch.float16, n)
        check(lib().esp_route_rot(*args, suh0.data_ptr(), suh1.data_ptr(), out0.data_ptr(), out1.data_ptr(),
                                  int(e_tab), stream_ptr(x.device)))

    @staticmethod
    def group(pick, uids, ucount, members, R, slots, E):
        for t, n in ((pick, "pick"), (uids, "uids"), (ucount, "ucount"), (members, "members")):
            _check(t, torch.int32, n)
        _need(pick.numel() >= R * slots, "pick too small")
        _need(uids.numel() >= min(R * slots, E), "uids too small")
        check(lib().esp_group(pick.data_ptr(), R, slots, E, uids.data_ptr(), ucount.data_ptr(), members.data_ptr(),
                              members.size(1), uids.numel(), stream_ptr(pick.device)))

    @staticmethod
    def group_shared(pick_in, wts_in, x, x_stride, gate_w, shared_id, pick_out, wts_out, uids, ucount, members, R,
                     slots_in, E):
        _need(x.is_cuda and x.dtype in (torch.bfloat16, torch.float16), "x: bf16/fp16 CUDA")
        if gate_w is not None:
            _need(gate_w.dtype == x.dtype and gate_w.is_contiguous() and gate_w.numel() == x.size(1),
                  "gate_w: x's dtype, [H]")
        _need(shared_id < 0 or gate_w is not None, "a shared slot needs its gate weight")
        check(lib().esp_group_shared(pick_in.data_ptr(), wts_in.data_ptr(), x.data_ptr(), DTYPE[x.dtype], int(x_stride),
                                     x.size(1), ptr(gate_w), int(shared_id), pick_out.data_ptr(), wts_out.data_ptr(),
                                     uids.data_ptr(), ucount.data_ptr(), members.data_ptr(), R, slots_in, E,
                                     members.size(1), uids.numel(), stream_ptr(x.device)))

    @staticmethod
    def rot_in(x, x_stride, pick, suh0, suh1, out0, out1, rows, K, slots, E):
        _need(x.is_cuda and x.dtype in (torch.bfloat16, torch.float16), "x: bf16/fp16 CUDA")
        for t, n in ((suh0, "suh0"), (suh1, "suh1"), (out0, "out0"), (out1, "out1")):
            _check(t, torch.float16, n)
        check(lib().esp_rot_in(x.data_ptr(), DTYPE[x.dtype], int(x_stride), pick.data_ptr(), suh0.data_ptr(),
                               suh1.data_ptr(), out0.data_ptr(), out1.data_ptr(), rows, K, slots, E,
                               stream_ptr(x.device)))

    @staticmethod
    def grouped(X0, X1, TP0, TP1, B0, B1, C0, C1, uids, ucount, members, Z, mats, K, N, P, SK, slots, nt=4, warps=4,
                pf=2, lo=2, hi=16, tables=None):
        """nt / warps / pf / lo / hi are the reference's tile hints (accepted, unused). `tables` = host copies of the
        k2 / cb tables ([mats][E] each) so unsupported (codebook, width) pairs are refused on the host; if omitted they
        are read back from the device tables (a synchronisation)."""
        _check(X0, torch.float16, "X0")
        _check(Z, torch.float32, "Z")
        _need(Z.numel() >= mats * SK * P * N, "Z too small")
        E = TP0.numel()
        if tables is None:
            k2h = torch.cat([B0.cpu(), B1.cpu()] if mats == 2 else [B0.cpu()]).to(torch.int32).contiguous()
            cbh = torch.cat([C0.cpu(), C1.cpu()] if mats == 2 else [C0.cpu()]).to(torch.int32).contiguous()
        else:
            k2h, cbh = tables
        check(lib().esp_grouped(X0.data_ptr(), X1.data_ptr(), TP0.data_ptr(), TP1.data_ptr(), B0.data_ptr(),
                                B1.data_ptr(), C0.data_ptr(), C1.data_ptr(), k2h.data_ptr(), cbh.data_ptr(), E,
                                uids.data_ptr(), ucount.data_ptr(), members.data_ptr(), uids.numel(), members.size(1),
                                Z.data_ptr(), mats, K, N, P, SK, slots, stream_ptr(X0.device)))

    @staticmethod
    def gateup_epilogue(Z, pick, svh_g, svh_u, suh_d, xd, rows, P, N, SK, slots, E, limit, act_mode):
        _check(Z, torch.float32, "Z")
        for t, n in ((svh_g, "svh_g"), (svh_u, "svh_u"), (suh_d, "suh_d"), (xd, "xd")):
            _check(t, torch.float16, n)
        lim = float(limit) if limit != float("inf") else float("inf")
        check(lib().esp_gateup_epilogue(Z.data_ptr(), pick.data_ptr(), svh_g.data_ptr(), svh_u.data_ptr(),
                                        suh_d.data_ptr(), xd.data_ptr(), rows, P, N, SK, slots, E, lim, int(act_mode),
                                        stream_ptr(Z.device)))

    @staticmethod
    def down_epilogue(Z, pick, svh_d, y, rows, P, D, SK, slots, E):
        check(lib().esp_down_combine(Z.data_ptr(), pick.data_ptr(), svh_d.data_ptr(), y.data_ptr(), None, None, None,
                                     2, rows, P, D, SK, slots, E, slots, 0, stream_ptr(Z.device)))

    @staticmethod
    def combine(y, wts, out, rows, D, slots):
        check(lib().esp_combine(y.data_ptr(), wts.data_ptr(), out.data_ptr(), rows, D, slots, stream_ptr(y.device)))

    @staticmethod
    def down_combine(Z, pick, svh_d, y, wts, out, rows, P, D, SK, slots, E):
        _check(out, torch.float32, "out")
        check(lib().esp_down_combine(Z.data_ptr(), pick.data_ptr(), svh_d.data_ptr(), y.data_ptr(), wts.data_ptr(),
                                     out.data_ptr(), None, 2, rows, P, D, SK, slots, E, slots, 1, stream_ptr(Z.device)))

    @staticmethod
    def down_combine2(Z, pick, svh_d, y, wts, out, out_shared, rows, P, D, SK, slots, E, n_routed):
        _need(out.is_cuda and out.is_contiguous() and out.dtype in DTYPE, "out: contiguous CUDA")
        if out_shared is not None:
            _need(out_shared.dtype == out.dtype and out_shared.is_contiguous(), "out_shared: out's dtype")
        _need(n_routed <= slots, "n_routed <= slots")
        check(lib().esp_down_combine(Z.data_ptr(), pick.data_ptr(), svh_d.data_ptr(), y.data_ptr(), wts.data_ptr(),
                                     out.data_ptr(), ptr(out_shared), DTYPE[out.dtype], rows, P, D, SK, slots, E,
                                     int(n_routed), 1, stream_ptr(Z.device)))

    # ---- the fused B200 pipeline (no reference counterpart: replaces grouped + epilogues) ----
    @staticmethod
    def moe_gateup(xg, xu, L, uids, ucount, members, slots, P, S, z, counters, xd):
        k2h, cbh = L.host_tables("gu")
        g, u, d = L.gate, L.up, L.down
        check(lib().esp_moe_gateup(xg.data_ptr(), xu.data_ptr(), g.ptr.data_ptr(), u.ptr.data_ptr(), g.k2.data_ptr(),
                                   u.k2.data_ptr(), g.cb.data_ptr(), u.cb.data_ptr(), k2h.data_ptr(), cbh.data_ptr(),
                                   L.E, g.svh.data_ptr(), u.svh.data_ptr(), d.suh.data_ptr(), uids.data_ptr(),
                                   ucount.data_ptr(), members.data_ptr(), uids.numel(), members.size(1), slots, P, L.D,
                                   L.I, S, z.data_ptr(), counters.data_ptr(), xd.data_ptr(), stream_ptr(xg.device)))

    @staticmethod
    def moe_layer(xg, xu, L, uids, ucount, members, pick, wts, slots, n_routed, rows, S, z, xd, y, counters, out,
                  out_shared):
        k2h, cbh = L.host_tables("all")
        g, u, d = L.gate, L.up, L.down
        check(lib().esp_moe_layer(xg.data_ptr(), xu.data_ptr(), g.ptr.data_ptr(), u.ptr.data_ptr(), d.ptr.data_ptr(),
                                  g.k2.data_ptr(), u.k2.data_ptr(), d.k2.data_ptr(), g.cb.data_ptr(), u.cb.data_ptr(),
                                  d.cb.data_ptr(), k2h.data_ptr(), cbh.data_ptr(), L.E, g.svh.data_ptr(),
                                  u.svh.data_ptr(), d.suh.data_ptr(), d.svh.data_ptr(), uids.data_ptr(),
                                  ucount.data_ptr(), members.data_ptr(), uids.numel(), members.size(1),
                                  pick.data_ptr(), wts.data_ptr(), slots, int(n_routed), rows, L.D, L.I, int(S),
                                  z.data_ptr(), xd.data_ptr(), y.data_ptr(), counters.data_ptr(), out.data_ptr(),
                                  ptr(out_shared), DTYPE[out.dtype], stream_ptr(xg.device)))

    @staticmethod
    def moe_layer_ep(xg, xu, L, uids, ucount, members, local_pick, no_w, slots, rows, S, z, xd, counters, inbox_y,
                     flags_y, epoch, world, rank, R, scratch_out):
        """esp_moe_layer for the expert-parallel layer: y rows into their home ranks' inboxes (inbox_y / flags_y:
        ctypes arrays of every rank's addresses), flags released by the launch."""
        k2h, cbh = L.host_tables("all")
        g, u, d = L.gate, L.up, L.down
        check(lib().esp_moe_layer_ep(xg.data_ptr(), xu.data_ptr(), g.ptr.data_ptr(), u.ptr.data_ptr(), d.ptr.data_ptr(),
                                     g.k2.data_ptr(), u.k2.data_ptr(), d.k2.data_ptr(), g.cb.data_ptr(),
                                     u.cb.data_ptr(), d.cb.data_ptr(), k2h.data_ptr(), cbh.data_ptr(), L.E,
                                     g.svh.data_ptr(), u.svh.data_ptr(), d.suh.data_ptr(), d.svh.data_ptr(),
                                     uids.data_ptr(), ucount.data_ptr(), members.data_ptr(), uids.numel(),
                                     members.size(1), local_pick.data_ptr(), no_w.data_ptr(), slots, rows, L.D, L.I,
                                     int(S), z.data_ptr(), xd.data_ptr(), counters.data_ptr(), inbox_y, flags_y,
                                     epoch, world, rank, R, scratch_out.data_ptr(), stream_ptr(xg.device)))

    @staticmethod
    def moe_down(xd, L, uids, ucount, members, pick, wts, slots, n_routed, rows, y, counters, out, out_shared):
        k2h, cbh = L.host_tables("d")
        d = L.down
        check(lib().esp_moe_down(xd.data_ptr(), d.ptr.data_ptr(), d.k2.data_ptr(), d.cb.data_ptr(), k2h.data_ptr(),
                                 cbh.data_ptr(), L.E, d.svh.data_ptr(), uids.data_ptr(), ucount.data_ptr(),
                                 members.data_ptr(), uids.numel(), members.size(1), pick.data_ptr(), wts.data_ptr(),
                                 slots, int(n_routed), rows, L.I, L.D, y.data_ptr(), counters.data_ptr(),
                                 out.data_ptr(), ptr(out_shared), DTYPE[out.dtype], stream_ptr(xd.device)))


@lru_cache(1)
def ext() -> _Ext:
    lib()
    return _Ext()


def device_status(reset: bool = True) -> int:
    v = C.c_int(0)
    check(lib().esp_device_status(C.byref(v), int(reset)))
    return v.value
