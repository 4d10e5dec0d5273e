"""Expert parallelism host logic on CPU ranks (gloo, world sizes 2, 4 and 8): the dispatch / local-table / give-back path of
vllm_espalier_b200.ep with a stand-in expert function must deliver every routed slot's y row to its home rank, so that
the slot-ordered combine gives the same bits as one process holding every expert.

The stand-in writes NaN wherever a rank computes a (row, slot) that is not its own, so a y row taken from the wrong rank
or slot shows up in the output."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O

E, K, R, D = 16, 4, 5, 128


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(rank: int):
    g = torch.Generator().manual_seed(1000 + rank)
    x = torch.randn(R, D, generator=g).to(torch.bfloat16)
    pick = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(R)]).to(torch.int32)
    pick[1, 2] = -1                                                     # a skipped slot
    pick = torch.cat([pick, torch.full((R, 1), E, dtype=torch.int32)], 1)   # the shared slot, id E
    wts = torch.rand(R, K + 1, generator=g).to(torch.float32)
    return x, pick, wts


def _expert(xrow: torch.Tensor, e: int) -> torch.Tensor:
    """Stand-in for an expert's fp32 output row."""
    return (xrow.float() * (e + 1) / 7.0 + 0.25 * e).to(torch.float32)


def _combine(y_of, pick: torch.Tensor, wts: torch.Tensor):
    """Slot-ordered fp32 fma combine (the kernels' arithmetic, through the C oracle) and the shared slot's w * y."""
    out = np.zeros((R, D), np.float32)
    sh = np.zeros((R, D), np.float32)
    for r in range(R):
        js = [j for j in range(K) if 0 <= int(pick[r, j]) < E]
        if js:
            ys = np.stack([y_of(r, j) for j in js])
            out[r] = O.combine_row(ys, wts[r, js].numpy(), len(js))
        sh[r] = wts[r, K].numpy() * y_of(r, K)
    return out, sh


def _worker(rank: int, world: int, port: int, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import __graft_entry__
        __graft_entry__.load_package()
        from vllm_espalier_b200 import ep
        x, pick, wts = _inputs(rank)
        recv_x, recv_p = ep.dispatch(x, pick, world)
        lp = ep.local_table(recv_p, rank, world, E, K)
        e0, e1 = ep.expert_range(rank, world, E)
        y = torch.full((world, R, K + 1, D), float("nan"), dtype=torch.float32)
        for s in range(world):
            for r in range(R):
                for j in range(K + 1):
                    le = int(lp[s, r, j])
                    if le < 0:
                        continue
                    ge = E if le == e1 - e0 else e0 + le          # the local shared entry is nl
                    y[s, r, j] = _expert(recv_x[s, r], ge)
        back = ep.give_back(y)
        owner = ep.owner_of(pick.long().clamp(min=0), world, E)

        def y_ep(r, j):
            src = rank if j == K else int(owner[r, j])
            return back[src, r, j].numpy()

        def y_one(r, j):
            return _expert(x[r], int(pick[r, j])).numpy()
        got = _combine(y_ep, pick, wts)
        want = _combine(y_one, pick, wts)
        ok = all(np.array_equal(a.view(np.uint32), b.view(np.uint32)) for a, b in zip(got, want))
        q.put((rank, ok, bool(np.isfinite(got[0]).all() and np.isfinite(got[1]).all())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_exchange_matches_one_rank_bitwise(world):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    res = sorted(q.get() for _ in range(world))
    assert all(ok and finite for _, ok, finite in res), res


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_expert_ranges_partition_and_owner(world):
    from vllm_espalier_b200 import ep
    ranges = [ep.expert_range(q, world, 256) for q in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == 256
    assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    e = torch.arange(256)
    own = ep.owner_of(e, world, 256)
    for q, (e0, e1) in enumerate(ranges):
        assert bool((own[e0:e1] == q).all())


def test_local_table_marks_only_own_experts_and_own_shared_slot():
    from vllm_espalier_b200 import ep
    world, E_, k = 2, 8, 2
    recv = torch.tensor([[[0, 5, E_], [7, 3, E_]], [[4, 1, E_], [-1, 6, E_]]], dtype=torch.int32)  # [world][R=2][3]
    lp1 = ep.local_table(recv, 1, world, E_, k)          # rank 1 holds experts 4..7, local shared id 4
    assert lp1.tolist() == [[[-1, 1, -1], [3, -1, -1]], [[0, -1, 4], [-1, 2, 4]]]
    lp0 = ep.local_table(recv, 0, world, E_, k)
    assert lp0.tolist() == [[[0, -1, 4], [-1, 3, 4]], [[-1, 1, -1], [-1, -1, -1]]]
