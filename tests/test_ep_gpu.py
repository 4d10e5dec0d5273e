"""Expert-parallel MoE layer on 2, 4 and 8 GPUs, with either exchange (p2p: peer stores and flags, the default; nccl:
two all_to_all collectives): each rank's EPLayer output must equal, bit for bit, the single-GPU fused path (route +
routed2) on a layer holding every expert, for the same rows, on two calls in a row (the second runs on the advanced
epoch and the inboxes the first left). Each world size is skipped on a box with fewer GPUs.

One case biases the router so that one expert is picked by every row: the 32 rows of every rank then give that expert
32 x world members, more than a grouping entry holds (32), which exercises the chunked grouping."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

import cases as C

pytestmark = pytest.mark.gpu
GRID_OF = {1: 0, 3: 1, 6: 3, 7: 4}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _Mat:
    def __init__(self, T, K, cb, suh, svh, dev):
        self.trellis = torch.from_numpy(np.ascontiguousarray(T)).to(dev)
        self.suh = torch.from_numpy(suh).to(dev)
        self.svh = torch.from_numpy(svh).to(dev)
        self.K, self.cb = K, GRID_OF[cb]
        self.in_features, self.out_features = T.shape[0] * 16, T.shape[1] * 16


def _bf(a_bits, dev):
    return torch.from_numpy(np.ascontiguousarray(a_bits).view(np.int16)).to(dev).view(torch.bfloat16)


def _worker(rank, world, port, R, bias, exchange, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), ESPALIER_EP_EXCHANGE=exchange)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        import __graft_entry__
        __graft_entry__.load_package()
        from vllm_espalier_b200 import ep
        from vllm_espalier_b200 import experts as G
        experts_np, _, _, _, gate_w = C.moe_inputs()
        E, D, k = C.MOE_E, C.MOE_D, C.MOE_K
        r = C.rng("ep-router")
        gate = (r.standard_normal((E, D)) / np.sqrt(D)).astype(np.float32)
        if bias:
            gate[0] *= 40.0
        gate_b = _bf(C.bf16_bits(gate), dev)
        x = _bf(C.activations(("ep-x", rank, R), R, D), dev)

        def mats():
            return [tuple(_Mat(*ex[p], dev) for p in ("gate", "up", "down")) for ex in experts_np]
        full = mats()
        L = G.prepare(full[:-1], full[-1], _bf(gate_w, dev))
        s = G.scratch(L, 32, k + 1, dev)
        G.route(x, gate_b, k, L, s)
        want, want_sh = G.routed2(x, None, None, L, s, k=k)

        e0, e1 = ep.expert_range(rank, world, E)
        mine = mats()
        epl = ep.EPLayer(mine[e0:e1], mine[-1], _bf(gate_w, dev), rank, world, E, rows=32, k=k)
        assert epl.exchange == exchange
        same = True
        for _ in range(2):
            got, got_sh = epl.forward(x, gate_b)
            torch.cuda.synchronize()
            same &= bool(torch.equal(got, want)) and bool(torch.equal(got_sh, want_sh))
        n_entries = int(epl.count.item())
        from vllm_espalier_b200 import _lib
        status = _lib.device_status()
        dist.barrier()
        if epl.ex is not None:
            epl.ex.close()
        q.put((rank, same, status == 0, float((got.float() - want.float()).abs().max()), n_entries))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["p2p", "nccl"])
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("R,bias", [(3, False), (32, False), (32, True)])
def test_ep_bitwise_equal_to_one_gpu(world, R, bias, exchange):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(rk, world, port, R, bias, exchange, q)) for rk in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    res = sorted(q.get() for _ in range(world))
    assert all(a and b for _, a, b, _, _ in res), res
