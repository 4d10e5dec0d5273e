"""The bounded device waits' failure path, with no GPU fault: a wait on a flag that nothing sets gives up after its
time limit, records ESP_ERR_TIMEOUT in the status word the host reads (esp_device_status), and leaves the context
usable; a flag that is set is seen at once. The status is reset afterwards so later kernels wait their full limit."""
from __future__ import annotations

import time

import numpy as np
import pytest
import torch

import cases as C
import oracle as O
from helpers import f32, rel_err

from vllm_espalier_b200 import _lib
from vllm_espalier_b200 import dense as D

pytestmark = pytest.mark.gpu


def _wait(flag, need, result, dev):
    _lib.check(_lib.lib().esp_wait_flag(flag.data_ptr(), need, result.data_ptr(), _lib.stream_ptr(dev)))


def test_wait_on_unset_flag_times_out_and_context_survives(dev):
    _lib.device_status(reset=True)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    result = torch.full((1,), -1, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _wait(flag, 1, result, dev)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    try:
        assert int(result.item()) == 0, "the wait did not give up"
        assert waited >= 0.15, f"gave up after {waited:.3f} s, before its limit"
        assert _lib.device_status(reset=True) == _lib.ESP_ERR_TIMEOUT
    finally:
        _lib.device_status(reset=True)
    assert _lib.device_status(reset=False) == 0
    # a set flag is seen at once
    flag.fill_(3)
    _wait(flag, 3, result, dev)
    torch.cuda.synchronize()
    assert int(result.item()) == 1 and _lib.device_status(reset=False) == 0
    # the context still runs a layer correctly
    mats, xf = C.dense_inputs("wait", 512, [256], 7, 8, 4, "bf16")
    T, suh, svh = mats[0]
    m = type("M", (), {})()
    m.trellis, m.suh, m.svh = (torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in (T, suh, svh))
    m.K, m.cb, m.in_features, m.out_features = 4, 4, 512, 256
    y = D.Dense([m]).forward(torch.from_numpy(xf).to(dev).to(torch.bfloat16))
    assert rel_err(f32(y), O.dense_matrix(xf, T, suh, svh, 4, 7)) < 1e-2
    assert _lib.device_status(reset=False) == 0
