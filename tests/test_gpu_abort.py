"""GPU: the bounded-wait abort path, exercised without a fault.

Every device-side wait of the matmul kernels gives up after a wall-clock limit, records a
status bit and lets the kernel drain and return (the reference's MLX kernels have no
device-side waits; this is the library's own failure detection).  The testing hook
``sdq_debug_wait_hook`` shortens the limit and makes each CTA's weight producer withhold its
first copy and the arrival that goes with it -- a flag that nothing sets, from the
consumers' point of view -- so the wait on that stage runs out.  The tests check that

  * the call returns and the stream drains within a bound (no unbounded wait);
  * ``sdq_device_status`` reports SDQ_ERR_TIMEOUT with the kernel's bits, then clears;
  * the next call, with the hook off, is correct (the context and the kernel's state are
    intact: barriers, tensor memory, status words).
"""
from __future__ import annotations

import time

import numpy as np
import pytest
import torch

import oracle as O
import sdq
from conftest import gpu_available
from sdq import _abi

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not gpu_available(), reason="needs an sm_100 device")]

LIMIT_NS = 20_000_000          # 20 ms: far above any wait of these sizes, far below 2 s


def bits16(t):
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


def check_result(y, xb, q, n, bits):
    want = O.qmatmul(xb, q.weight.cpu().numpy().view(np.uint32), bits16(q.scales), bits16(q.biases), n, bits)
    g, w = y.float().cpu().numpy().astype(np.float64), want.astype(np.float64)
    rel = float(np.max(np.abs(g - w)) / np.max(np.abs(w)))
    assert rel <= 1e-2 and O.cosine(w, g) >= 0.9999, rel


# m = 4: the small-M weight-stream kernel; m = 16: the tensor-core kernel with resident
# activations; m = 300: the tensor-core kernel with an activation ring.
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m", [4, 16, 300])
def test_withheld_copy_times_out_then_the_next_call_is_correct(bits, m):
    k, n = 1024, 512
    xb, w = O.synthetic_linear(60 + m + bits, m, k, n, 0.02)
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
    q = sdq.QuantizedArray.quantize(torch.from_numpy(w).cuda(), 64, bits)
    check_result(q.matmul(x), xb, q, n, bits)
    sdq.device_status()                                    # clean before

    sdq.debug_wait_hook(LIMIT_NS, True)
    try:
        t0 = time.monotonic()
        q.matmul(x)
        torch.cuda.synchronize()
        elapsed = time.monotonic() - t0
        with pytest.raises(sdq.SdqError) as e:
            sdq.device_status()
    finally:
        sdq.debug_wait_hook(0, False)
    assert e.value.code == _abi.SDQ_ERR_TIMEOUT and "gave up" in str(e.value)
    # each CTA waits out a handful of 20 ms limits (the stalled wait, then the drains)
    assert elapsed < 5.0, f"the aborted call took {elapsed:.2f} s"
    sdq.device_status()                                    # the status word was cleared

    y = q.matmul(x)
    sdq.device_status()
    check_result(y, xb, q, n, bits)


def test_hook_rejects_a_limit_out_of_range():
    for bad in (1, 999_999, 2_000_000_001):
        with pytest.raises(sdq.SdqError) as e:
            sdq.debug_wait_hook(bad, False)
        assert e.value.code == _abi.SDQ_ERR_INVALID
    sdq.debug_wait_hook(0, False)
