"""GPU parity of the trellis decode, the Hadamard kernel and the fused dense decode GEMV against the CPU oracle.

Gates (BASELINE.json north_star and the reference's tests/gpu_dense.py / gpu_grouped.py):
  * decoded weights bit-exact for every compiled (codebook, width) pair;
  * had bit-exact;
  * dense layer outputs within max rel err 1e-2 of the oracle (the north_star bar) and within the output-rounding
    floor + 2e-3 (a much tighter check);
  * rows alone == rows in the window, merged launch == each matrix alone, CUDA graph replay == eager (bit for bit);
  * the split-K counters are left zero, no device-side timeout.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import cases as C
import oracle as O
from helpers import bits, f32, floor_err, rel_err, to_dev

from vllm_espalier_b200 import _lib
from vllm_espalier_b200 import dense as D
from vllm_espalier_b200.experts import dequant

pytestmark = pytest.mark.gpu
GRID_OF = {1: 0, 3: 1, 6: 3, 7: 4}   # kernel cb -> Espalier grid code


class Mat:
    def __init__(self, T, suh, svh, K, cb, dev):
        self.trellis = to_dev(T, dev)
        self.suh = to_dev(suh, dev)
        self.svh = to_dev(svh, dev)
        self.K, self.cb = K, GRID_OF[cb]
        self.in_features, self.out_features = T.shape[0] * 16, T.shape[1] * 16


@pytest.mark.parametrize("cb,k2", C.COMPILED)
def test_dequant_bit_exact(dev, cb, k2):
    T = C.dequant_case(cb, k2)
    got = bits(dequant(to_dev(T, dev), k2 // 2, GRID_OF[cb]))
    want = O.bits16(O.dequant(T, k2 // 2, cb))
    assert np.array_equal(got, want), f"{int((got != want).sum())} weights differ"


@pytest.mark.parametrize("cb,k2", [(1, 16), (3, 6), (6, 8), (7, 10), (3, 2)])
def test_dequant_bit_exact_large(dev, cb, k2):
    """A 512 x 1024 matrix: 2048 tiles, every lane position and word alignment many times over."""
    T = C.trellis(("dq-large", cb, k2), 512, 1024, k2 // 2)
    got = bits(dequant(to_dev(T, dev), k2 // 2, GRID_OF[cb]))
    want = O.bits16(O.dequant(T, k2 // 2, cb))
    assert np.array_equal(got, want), f"{int((got != want).sum())} weights differ"


def test_had_bit_exact(dev):
    x, pre, post = C.had_case()
    y = torch.empty(x.shape, dtype=torch.float16, device=dev)
    _lib.ext().had(to_dev(x, dev), to_dev(pre, dev), to_dev(post, dev), y)
    assert np.array_equal(bits(y), O.bits16(O.had(x, pre, post)))
    _lib.ext().had(to_dev(x, dev), None, None, y)
    assert np.array_equal(bits(y), O.bits16(O.had(x)))


def _layer(name, K, Ns, cb, k2, M, xdt, dev):
    mats, xf = C.dense_inputs(name, K, Ns, cb, k2, M, xdt)
    ms = [Mat(T, su, sv, k2 // 2, cb, dev) for T, su, sv in mats]
    tdt = torch.bfloat16 if xdt == "bf16" else torch.float16
    ref = np.concatenate([O.dense_matrix(xf, T, su, sv, k2 // 2, cb) for T, su, sv in mats], axis=1)
    return ms, torch.from_numpy(xf).to(dev).to(tdt), ref


CASES = [(n, K, Ns, cb, k2, M, xdt) for n, K, Ns, cb, k2, Ms, xdt in C.DENSE_CASES for M in Ms]


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}-M{c[5]}" for c in CASES])
def test_dense_vs_oracle(dev, case):
    ms, x, ref = _layer(*case, dev)
    y = D.Dense(ms).forward(x)
    torch.cuda.synchronize()
    e, fl = rel_err(f32(y), ref), floor_err(ref, y.dtype)
    assert e < 1e-2, f"max rel err {e:.3e}"
    assert e < fl + 2e-3, f"max rel err {e:.3e} vs rounding floor {fl:.3e}"
    assert _lib.device_status() == 0


@pytest.mark.parametrize("M", [1, 8, 32])
def test_config2_block_vs_oracle(dev, M):
    """q/k/v (2048 -> 4096 + 512 + 512) merged, and o (4096 -> 2048), 4-bit int5."""
    qkv, x, ref = _layer("cfg2-qkv", 2048, [4096, 512, 512], 6, 8, M, "bf16", dev)
    y = D.Dense(qkv).forward(x)
    o, xo, ref_o = _layer("cfg2-o", 4096, [2048], 6, 8, M, "bf16", dev)
    yo = D.Dense(o).forward(xo)
    torch.cuda.synchronize()
    for got, want in ((y, ref), (yo, ref_o)):
        e, fl = rel_err(f32(got), want), floor_err(want, got.dtype)
        assert e < 1e-2 and e < fl + 2e-3, f"max rel err {e:.3e} (floor {fl:.3e})"


@pytest.mark.parametrize("M", [1, 8, 32])
def test_config1_layer_vs_oracle(dev, M):
    """BASELINE config 1's exact shape: one 2048 -> 4096 matrix, 4-bit trellis, int6 codebook (kernel codebook 7)."""
    ms, x, ref = _layer("cfg1", 2048, [4096], 7, 8, M, "bf16", dev)
    y = D.Dense(ms).forward(x)
    torch.cuda.synchronize()
    e, fl = rel_err(f32(y), ref), floor_err(ref, y.dtype)
    assert e < 1e-2 and e < fl + 2e-3, f"max rel err {e:.3e} (floor {fl:.3e})"
    assert _lib.device_status() == 0
    assert int(D.workspace(dev).counters.abs().sum()) == 0


@pytest.mark.parametrize("M", [1, 17])
def test_wide_layer_vs_oracle(dev, M):
    """A layer with more 128-column blocks (240) than SMs: one range an SM over whole blocks with a partial block at
    each end, finished through global partial sums by the last CTA to arrive (the path a narrow layer's clusters
    avoid); 6-bit mcg as the LM head uses."""
    ms, x, ref = _layer("wide", 256, [240 * 128], 1, 12, M, "bf16", dev)
    y = D.Dense(ms).forward(x)
    torch.cuda.synchronize()
    e, fl = rel_err(f32(y), ref), floor_err(ref, y.dtype)
    assert e < 1e-2 and e < fl + 2e-3, f"max rel err {e:.3e} (floor {fl:.3e})"
    assert _lib.device_status() == 0


def test_rows_alone_equal_window(dev):
    ms, x, _ = _layer("int5_3bit", 512, [128, 128], 6, 6, 17, "bf16", dev)
    d = D.Dense(ms)
    win = d.forward(x).clone()
    for r in range(x.shape[0]):
        alone = d.forward(x[r:r + 1].contiguous())
        assert torch.equal(alone[0], win[r]), f"row {r} differs alone"
    for M in (2, 8, 9):
        part = d.forward(x[:M].contiguous())
        assert torch.equal(part, win[:M])


def test_merged_equals_alone(dev):
    ms, x, _ = _layer("int5_qkv", 256, [256, 128, 128], 6, 8, 5, "bf16", dev)
    merged = D.Dense(ms).forward(x)
    c = 0
    for m in ms:
        alone = D.Dense([m]).forward(x)
        assert torch.equal(alone, merged[:, c:c + m.out_features])
        c += m.out_features


def test_graph_equals_eager_and_scratch_zero(dev):
    """Graph replay gives the eager bits, and the scratch the kernel shares between launches (the tagged split-K
    partials, the counters) is left zero by every launch."""
    ms, x, _ = _layer("int6_single", 512, [256], 7, 8, 8, "bf16", dev)
    d = D.Dense(ms)
    eager = d.forward(x).clone()
    out = torch.empty_like(eager)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        d.forward(x, out=out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        d.forward(x, out=out)
    out.zero_()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    assert int(d.ws.counters.abs().sum()) == 0
    assert not bool(d.ws.z.view(torch.int32).any())


def test_fp32_and_fp16_io(dev):
    ms, x, ref = _layer("e2m1_2bit", 256, [128], 3, 4, 3, "fp16", dev)
    d = D.Dense(ms)
    for dt in (torch.float32, torch.float16):
        y = d.forward(x.to(dt))
        assert y.dtype == dt
        assert rel_err(f32(y), ref) < 2e-3


def test_errors_are_raised(dev):
    ms, x, _ = _layer("int6_single", 512, [256], 7, 8, 1, "bf16", dev)
    d = D.Dense(ms)
    z, xh = d.ws.z, d.ws.xh
    y = torch.empty((1, 256), dtype=torch.bfloat16, device=dev)
    with pytest.raises(RuntimeError, match="unsupported codebook"):
        _lib.ext().dense(x, [ms[0].trellis], [ms[0].suh], [ms[0].svh], [0], y, xh, z, d.ws.counters, 8, 3)
    with pytest.raises(RuntimeError, match="1 to 32 rows"):
        big = torch.zeros((33, 512), dtype=torch.bfloat16, device=dev)
        _lib.ext().dense(big, [ms[0].trellis], [ms[0].suh], [ms[0].svh], [0], y, xh, z, d.ws.counters, 8, 7)
