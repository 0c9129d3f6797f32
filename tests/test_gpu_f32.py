"""GPU: the f32 forms of the boundary (the reference's own tensors are f32).

MLX hands ``mlx_quantize`` an f32 weight and gets f32 scales and biases back; its
activations and the matmul's result are f32 too (crates/sd-tensor/src/mlx.rs:1861-1975).
libsdq accepts those dtypes at the C ABI:

  * f32 scales/biases from the quantiser hold the bf16 rule's values widened exactly, so
    they equal the bf16 tensors bit for bit after widening;
  * f32 scales passed to the dequantiser / matmul are rounded to bf16 (a no-op for the
    quantiser's own), so every result equals the bf16-scale call's bit for bit;
  * f32 activations are rounded to bf16 (nearest even) before the product, so the result
    equals the call with bf16(X) bit for bit, and stays within the parity bar of the f64
    product with the unrounded f32 X;
  * an f32 result is the kernel's f32 accumulator (plus bias), so rounding it to bf16 gives
    the bf16 call's result bit for bit.
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

MAX_ABS_REL = 1e-2
MIN_COSINE = 0.9999


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


def bits32(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy().view(np.uint32)


def rne_bf16(t: torch.Tensor) -> np.ndarray:
    """bf16 bits of an f32 device tensor, rounded to nearest even by the oracle."""
    return O.f32_to_bf16_bits(t.detach().cpu().numpy())


def weight(seed, n, k):
    return O.seeded_normals(seed, n * k).reshape(n, k) * np.float32(0.02)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("wdtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,k", [(256, 512), (3, 192), (129, 3072)])
def test_quantize_f32_scales_are_the_widened_bf16_ones(bits, wdtype, n, k):
    w = torch.from_numpy(weight(n + 3 * k, n, k)).cuda().to(wdtype)
    wq16, s16, b16 = sdq.quantize(w, 64, bits)
    wq32, s32, b32 = sdq.quantize(w, 64, bits, sb_dtype=torch.float32)
    assert s32.dtype == torch.float32 and b32.dtype == torch.float32
    assert torch.equal(wq16, wq32), "packed words"
    assert (bits32(s32) == bits16(s16).astype(np.uint32) << 16).all(), "scales"
    assert (bits32(b32) == bits16(b16).astype(np.uint32) << 16).all(), "biases"
    # and the oracle agrees with both
    rwq, rs, rb = O.quantize(w.float().cpu().numpy() if wdtype == torch.float32
                             else bits16(w), bits)
    assert (bits16(s16) == rs).all() and (wq16.cpu().numpy().view(np.uint32) == rwq).all()


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_dequantize_with_f32_scales_equals_bf16_scales(bits, out_dtype):
    n, k = 200, 1024
    w = torch.from_numpy(weight(11 + bits, n, k)).cuda()
    wq, s16, b16 = sdq.quantize(w, 64, bits)
    _, s32, b32 = sdq.quantize(w, 64, bits, sb_dtype=torch.float32)
    d16 = sdq.dequantize(wq, s16, b16, 64, bits, out_dtype=out_dtype)
    d32 = sdq.dequantize(wq, s32, b32, 64, bits, out_dtype=out_dtype)
    assert torch.equal(d16, d32)


def test_f32_scales_that_are_not_bf16_values_are_rounded():
    """An f32 scale outside the bf16 grid is rounded to nearest even, as the matmul's
    tensor-core operands are: dequantising with it equals dequantising with bf16(s)."""
    n, k, bits = 64, 256, 4
    w = torch.from_numpy(weight(5, n, k)).cuda()
    wq, s16, b16 = sdq.quantize(w, 64, bits)
    g = torch.Generator().manual_seed(3)
    s32 = (s16.float().cpu() * (1 + 1e-3 * torch.rand(s16.shape, generator=g))).cuda()
    b32 = (b16.float().cpu() * (1 + 1e-3 * torch.rand(b16.shape, generator=g))).cuda()
    sr = torch.from_numpy(rne_bf16(s32).view(np.int16)).cuda().view(torch.bfloat16)
    br = torch.from_numpy(rne_bf16(b32).view(np.int16)).cuda().view(torch.bfloat16)
    assert torch.equal(sdq.dequantize(wq, s32, b32, 64, bits, out_dtype=torch.bfloat16),
                       sdq.dequantize(wq, sr, br, 64, bits))
    assert sdq.dequantize(wq, s32, b32, 64, bits).dtype == torch.float32    # the scales' dtype
    x = torch.randn(20, k, generator=g).cuda().to(torch.bfloat16)
    assert torch.equal(sdq.quantized_matmul(x, wq, s32, b32, 64, bits),
                       sdq.quantized_matmul(x, wq, sr, br, 64, bits))


# Small-M weight stream (m <= 8) and the tensor-core kernel (every other m).
MS = [1, 3, 8, 9, 16, 300]


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m", MS)
@pytest.mark.parametrize("with_bias", [False, True])
def test_f32_result_rounds_to_the_bf16_result(bits, m, with_bias):
    k, n = 3072, 384
    xb, w = O.synthetic_linear(900 + m + bits, m, k, n, 0.02)
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
    q = sdq.QuantizedArray.quantize(torch.from_numpy(w).cuda(), 64, bits)
    bias16 = bias32 = None
    if with_bias:
        bias16 = torch.from_numpy(O.f32_to_bf16_bits(O.seeded_normals(m, n) * np.float32(0.5))
                                  .view(np.int16)).cuda().view(torch.bfloat16)
        bias32 = bias16.float()
    y16 = q.matmul(x, bias=bias16)
    y32 = q.matmul(x, bias=bias32, out=torch.empty(m, n, device="cuda", dtype=torch.float32))
    sdq.device_status()
    assert (rne_bf16(y32) == bits16(y16)).all()
    want = O.qmatmul(xb, q.weight.cpu().numpy().view(np.uint32), bits16(q.scales), bits16(q.biases), n,
                     bits, None if bias16 is None else bits16(bias16))
    g, wv = y32.cpu().numpy().astype(np.float64), want.astype(np.float64)
    rel = float(np.max(np.abs(g - wv)) / np.max(np.abs(wv)))
    assert rel <= MAX_ABS_REL and O.cosine(wv, g) >= MIN_COSINE, rel


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m", MS + [4096])
def test_f32_activations_and_scales(bits, m):
    """The reference's dtypes end to end: f32 X, f32 scales/biases, f32 Y."""
    k, n = 3072, 256
    vals = O.seeded_normals(4000 + m, m * k)
    x32 = vals.reshape(m, k).astype(np.float32)
    w = weight(77 + bits, n, k)
    q32 = sdq.QuantizedArray.quantize(torch.from_numpy(w).cuda(), 64, bits, sb_dtype=torch.float32)
    q16 = sdq.QuantizedArray.quantize(torch.from_numpy(w).cuda(), 64, bits)
    xd = torch.from_numpy(x32).cuda()
    y = q32.matmul(xd)
    sdq.device_status()
    assert y.dtype == torch.float32 and y.shape == (m, n)
    # bit-exact against the all-bf16-input call on bf16(X)
    xr = torch.from_numpy(O.f32_to_bf16_bits(x32).view(np.int16)).cuda().view(torch.bfloat16)
    yr = q16.matmul(xr, out=torch.empty(m, n, device="cuda", dtype=torch.float32))
    assert torch.equal(y, yr)
    # and within the parity bar of the f64 product with the UNROUNDED f32 activations
    rows = np.arange(m) if m <= 300 else np.linspace(0, m - 1, 97).astype(np.int64)
    dq = O.bf16_bits_to_f32(O.dequantize(q16.weight.cpu().numpy().view(np.uint32), bits16(q16.scales),
                                         bits16(q16.biases), n, k, bits)).astype(np.float64)
    want = x32[rows].astype(np.float64) @ dq.T
    g = y.cpu().numpy()[rows].astype(np.float64)
    rel = float(np.max(np.abs(g - want)) / np.max(np.abs(want)))
    assert rel <= MAX_ABS_REL and O.cosine(want, g) >= MIN_COSINE, rel


@pytest.mark.parametrize("bits", [4, 8])
def test_mixed_dtypes(bits):
    """bf16 X with f32 scales, f32 X with bf16 scales and a bf16 result: each equals the
    all-bf16 call on the rounded inputs."""
    m, k, n = 40, 1024, 192
    x32 = O.seeded_normals(41, m * k).reshape(m, k)
    w = torch.from_numpy(weight(42, n, k)).cuda()
    wq, s16, b16 = sdq.quantize(w, 64, bits)
    _, s32, b32 = sdq.quantize(w, 64, bits, sb_dtype=torch.float32)
    xr = torch.from_numpy(O.f32_to_bf16_bits(x32).view(np.int16)).cuda().view(torch.bfloat16)
    base = sdq.quantized_matmul(xr, wq, s16, b16, 64, bits)
    assert torch.equal(sdq.quantized_matmul(xr, wq, s32, b32, 64, bits), base)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    assert torch.equal(sdq.quantized_matmul(torch.from_numpy(x32).cuda(), wq, s16, b16, 64, bits, out=out),
                       base)


def test_fused_epilogue_stays_bf16():
    m, k, n = 16, 256, 128
    w = torch.from_numpy(weight(9, n, k)).cuda()
    wq, s, b = sdq.quantize(w, 64, 4)
    x = torch.randn(m, k, device="cuda")
    with pytest.raises(sdq.SdqError) as e:
        sdq.quantized_matmul_epilogue(x, wq, s, b, 64, 4, act="silu")
    assert e.value.code == _abi.SDQ_ERR_UNSUPPORTED and "bf16" in str(e.value)
