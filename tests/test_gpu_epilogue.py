"""GPU parity of the fused output stage, sdq_quantized_matmul_epilogue:
y = residual + gate * act(x . dequant(w)^T + bias), against the oracle (f64 product of the
dequantised weight, then the reference's chain in f64).

Shapes cover both kernels and every output path of each: the small-M weight stream (M <= 8),
the tensor-core kernel with resident activations (M <= 16), its 64 / 128-token tiles and the
wave-sized tall tiles, the TMA residual copy (N % 8 == 0) and the per-thread residual loads
(N % 8 != 0).  Bars as for the matmul: max-abs-rel <= 1e-2 and cosine >= 0.9999.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
import sdq
from conftest import gpu_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not gpu_available(), reason="needs an sm_100 device")]

MAX_ABS_REL = 1e-2
MIN_COSINE = 0.9999

SHAPES = [
    (1, 3072, 3072),     # small-M weight stream
    (5, 256, 36),        # weight stream, N not a multiple of 8
    (12, 1024, 512),     # tensor cores, activations resident
    (40, 512, 1000),     # 64-token tile, ragged N tile
    (17, 256, 36),       # 64-token tile, plain stores and per-thread residual loads
    (300, 512, 1024),    # 128-token tile... or taller, by the wave rule
    (1000, 3072, 3072),  # tall tiles (176 / 240 / 256 rows)
]

MODES = {
    "bias": dict(bias=True),
    "gelu": dict(bias=True, act=O.ACT_GELU_TANH),
    "silu": dict(act=O.ACT_SILU),
    "gate_residual": dict(bias=True, gate=True, residual=True),
    "everything": dict(bias=True, act=O.ACT_GELU_TANH, gate=True, residual=True),
}


def _bits16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


def _case(m, k, n, bits, seed):
    g = torch.Generator("cuda").manual_seed(seed)
    w = torch.randn(n, k, device="cuda", generator=g) * 0.02
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    bias = (torch.randn(n, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    gate = (torch.randn(n, device="cuda", generator=g)).to(torch.bfloat16)
    resid = (torch.randn(m, n, device="cuda", generator=g) * 2.0).to(torch.bfloat16)
    wq, s, b = sdq.quantize(w, 64, bits)
    return x, wq, s, b, bias, gate, resid


def _want(x, wq, s, b, n, bits, bias=None, act=O.ACT_NONE, gate=None, resid=None):
    acc = O.qmatmul(_bits16(x), wq.cpu().numpy().view(np.uint32), _bits16(s), _bits16(b), n, bits)
    return O.epilogue(acc, None if bias is None else _bits16(bias), act,
                      None if gate is None else _bits16(gate), None if resid is None else _bits16(resid))


def _check(got, want, what):
    g = got.float().cpu().numpy().astype(np.float64)
    rel = float(np.max(np.abs(g - want)) / max(np.max(np.abs(want)), 1e-30))
    cos = O.cosine(want, g)
    assert rel <= MAX_ABS_REL and cos >= MIN_COSINE, f"{what}: max-abs-rel {rel:.3e}, cosine {cos:.7f}"


@pytest.mark.parametrize("mode", sorted(MODES))
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m,k,n", SHAPES)
def test_fused_stage_matches_the_reference_chain(m, k, n, bits, mode):
    opt = MODES[mode]
    x, wq, s, b, bias, gate, resid = _case(m, k, n, bits, seed=m * 131 + n + bits)
    kw = dict(bias=bias if opt.get("bias") else None, act=opt.get("act", O.ACT_NONE),
              gate=gate if opt.get("gate") else None, residual=resid if opt.get("residual") else None)
    y = sdq.quantized_matmul_epilogue(x, wq, s, b, 64, bits, **kw)
    sdq.device_status()
    want = _want(x, wq, s, b, n, bits, kw["bias"], kw["act"], kw["gate"], kw["residual"])
    _check(y, want, f"{mode} m={m} k={k} n={n} W{bits}")


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m,k,n", [(3, 1024, 3072), (64, 512, 1000), (700, 3072, 3072), (17, 256, 36)])
def test_in_place_residual_update(m, k, n, bits):
    """out = residual: the Flux residual stream updated in place, x += gate * linear(a)."""
    x, wq, s, b, bias, gate, resid = _case(m, k, n, bits, seed=7 * m + n)
    want = _want(x, wq, s, b, n, bits, bias, O.ACT_NONE, gate, resid)
    stream = resid.clone()
    out = sdq.quantized_matmul_epilogue(x, wq, s, b, 64, bits, bias=bias, gate=gate, residual=stream,
                                        out=stream)
    sdq.device_status()
    assert out.data_ptr() == stream.data_ptr()
    _check(stream, want, f"in place m={m} n={n} W{bits}")


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m,k,n", [(1, 3072, 3072), (12, 1024, 512), (300, 512, 1024), (17, 256, 36)])
def test_bias_only_stage_equals_the_plain_matmul_bit_for_bit(m, k, n, bits):
    x, wq, s, b, bias, _, _ = _case(m, k, n, bits, seed=3 * m + n)
    plain = sdq.quantized_matmul(x, wq, s, b, 64, bits, bias=bias)
    fused = sdq.quantized_matmul_epilogue(x, wq, s, b, 64, bits, bias=bias)
    sdq.device_status()
    assert torch.equal(plain.view(torch.int16), fused.view(torch.int16))


def test_epilogue_argument_checks():
    x, wq, s, b, bias, gate, resid = _case(4, 256, 64, 4, seed=1)
    with pytest.raises(sdq.SdqError) as e:
        sdq.quantized_matmul_epilogue(x, wq, s, b, 64, 4, act="relu")
    assert e.value.code == sdq.SDQ_ERR_INVALID
    from sdq import _abi
    import ctypes
    y = torch.empty(4, 64, device="cuda", dtype=torch.bfloat16)
    rc = _abi.lib().sdq_quantized_matmul_epilogue(
        ctypes.c_void_p(x.data_ptr()), _abi.SDQ_BF16, 4, 256, ctypes.c_void_p(wq.data_ptr()),
        ctypes.c_void_p(s.data_ptr()), ctypes.c_void_p(b.data_ptr()), _abi.SDQ_BF16, 64, 64, 4, None, 7,
        None, None, ctypes.c_void_p(y.data_ptr()), _abi.SDQ_BF16,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _abi.SDQ_ERR_INVALID and "act must be" in _abi.last_error()
    big = torch.empty(8, 64, device="cuda", dtype=torch.bfloat16)
    rc = _abi.lib().sdq_quantized_matmul_epilogue(
        ctypes.c_void_p(x.data_ptr()), _abi.SDQ_BF16, 4, 256, ctypes.c_void_p(wq.data_ptr()),
        ctypes.c_void_p(s.data_ptr()), ctypes.c_void_p(b.data_ptr()), _abi.SDQ_BF16, 64, 64, 4, None, 0,
        None, ctypes.c_void_p(big[1:].data_ptr()), ctypes.c_void_p(big.data_ptr()), _abi.SDQ_BF16,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _abi.SDQ_ERR_INVALID and "overlaps" in _abi.last_error()
