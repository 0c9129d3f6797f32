"""GPU: sdq_quantized_matmul_host -- host activations in, host result out, row chunks
uploaded, multiplied and downloaded in overlap.

The pipeline must give exactly what the device entry point gives on the same row chunks
(the copies and the chunk bookkeeping add nothing), and within the parity bar of the oracle.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
import sdq
from conftest import gpu_available
from sdq import _abi

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not gpu_available(), reason="needs an sm_100 device")]


def bits16(t):
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


def pipe_chunks(m, asked):
    """Row counts of the chunks as the library picks them: the caller's size, else about
    m/8 rows (a multiple of 64, 128..1024); never more than 64 chunks."""
    r = asked if asked > 0 else min(max(((m + 7) // 8 + 63) // 64 * 64, 128), 1024)
    r = max(r, -(-m // 64))
    return [min(r, m - r0) for r0 in range(0, m, r)]


def chunked_device(x, q, rows, out_dtype, bias=None):
    """The device entry point on the same row chunks the pipeline uses."""
    ys, r0 = [], 0
    for r in rows:
        ys.append(sdq.quantized_matmul(x[r0:r0 + r].contiguous(), q.weight, q.scales, q.biases, 64, q.bits,
                                       bias=bias, out=torch.empty(r, q.weight.shape[0], device="cuda",
                                                                  dtype=out_dtype)))
        r0 += r
    return torch.cat(ys).cpu()


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m,chunk", [(4, 0), (300, 0), (300, 128), (1000, 128), (4096, 0), (4096, 512),
                                     (2051, 256)])
def test_host_pipeline_equals_device_chunks(bits, m, chunk):
    k, n = 1024, 384
    xb, w = O.synthetic_linear(500 + m + bits, m, k, n, 0.02)
    xh = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).pin_memory()
    q = sdq.QuantizedArray.quantize(torch.from_numpy(w).cuda(), 64, bits)
    y = sdq.quantized_matmul_host(xh, q.weight, q.scales, q.biases, 64, bits, chunk_rows=chunk)
    torch.cuda.synchronize()
    sdq.device_status()
    assert y.device.type == "cpu" and y.shape == (m, n) and y.dtype == torch.bfloat16
    assert torch.equal(y, chunked_device(xh.cuda(), q, pipe_chunks(m, chunk), torch.bfloat16))
    sample = np.arange(m) if m <= 300 else np.linspace(0, m - 1, 61).astype(np.int64)
    want = O.qmatmul(xb[sample], q.weight.cpu().numpy().view(np.uint32), bits16(q.scales), bits16(q.biases),
                     n, bits)
    g, wv = y.float().numpy()[sample].astype(np.float64), want.astype(np.float64)
    rel = float(np.max(np.abs(g - wv)) / np.max(np.abs(wv)))
    assert rel <= 1e-2 and O.cosine(wv, g) >= 0.9999, rel


def test_host_pipeline_f32_bias_and_pageable_memory():
    m, k, n, bits = 700, 512, 256, 4
    g = torch.Generator().manual_seed(7)
    x32 = torch.randn(m, k, generator=g)                      # pageable, f32
    w = torch.randn(n, k, generator=g) * 0.02
    q = sdq.QuantizedArray.quantize(w.cuda(), 64, bits, sb_dtype=torch.float32)
    bias = torch.randn(n, generator=g).cuda()
    y = sdq.quantized_matmul_host(x32, q.weight, q.scales, q.biases, 64, bits, bias=bias,
                                  out=torch.empty(m, n), chunk_rows=256)
    torch.cuda.synchronize()
    assert y.dtype == torch.float32
    assert torch.equal(y, chunked_device(x32.cuda(), q, pipe_chunks(m, 256), torch.float32, bias=bias))


def test_host_pipeline_runs_after_earlier_work_on_the_stream():
    """The call is ordered after what the caller queued before it on the same stream: a
    kernel still writing the host buffer's source must finish before the upload reads it."""
    m, k, n, bits = 2048, 1024, 512, 4
    q = sdq.QuantizedArray.quantize((torch.randn(n, k) * 0.02).cuda(), 64, bits)
    xd_src = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    xh = torch.empty(m, k, dtype=torch.bfloat16, pin_memory=True)
    xh.copy_(xd_src, non_blocking=True)                     # queued on the current stream
    y = sdq.quantized_matmul_host(xh, q.weight, q.scales, q.biases, 64, bits)
    torch.cuda.synchronize()
    ref = sdq.quantized_matmul(xd_src, q.weight, q.scales, q.biases, 64, bits)
    rel = float((y.float() - ref.float().cpu()).abs().max() / ref.float().abs().max())
    assert rel < 2e-2


def test_host_pipeline_rejects_device_buffers_as_host():
    m, k, n = 16, 128, 64
    q = sdq.QuantizedArray.quantize((torch.randn(n, k) * 0.02).cuda(), 64, 4)
    xd = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    yd = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    rc = _abi.lib().sdq_quantized_matmul_host(
        xd.data_ptr(), _abi.SDQ_BF16, m, k, q.weight.data_ptr(), q.scales.data_ptr(), q.biases.data_ptr(),
        _abi.SDQ_BF16, n, 64, 4, None, yd.data_ptr(), _abi.SDQ_BF16, xd.data_ptr(), yd.data_ptr(), 0,
        None)
    assert rc == _abi.SDQ_ERR_INVALID
    assert b"device memory" in _abi.lib().sdq_last_error()
