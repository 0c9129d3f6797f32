"""The CPU oracle, pinned: C restatement == independent NumPy restatement bit for bit,
the committed golden fixtures reproduce, and every threshold the reference's own
quantised-weight tests assert (crates/sd-models/tests/mlx_quantized.rs:53-228) holds
on the same deterministic inputs."""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "quantized_linear.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def _same(a, b):
    return a.shape == b.shape and (a == b).all()


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("shape,seed", [((256, 512), 1), ((3, 64), 2), ((17, 192), 3), ((64, 3072), 4)])
def test_c_and_numpy_quantise_agree(bits, shape, seed):
    n, k = shape
    w = O.seeded_normals(seed, n * k).reshape(n, k) * np.float32(0.02)
    a = O.quantize(w, bits)
    b = O.np_quantize(w, bits)
    assert all(_same(x, y) for x, y in zip(a, b))
    assert _same(O.dequantize(*a, n, k, bits), O.np_dequantize(*b, n, k, bits))


@pytest.mark.parametrize("bits", [4, 8])
def test_bf16_input_widens_exactly(bits):
    w = O.seeded_normals(7, 32 * 256).reshape(32, 256)
    wb = O.f32_to_bf16_bits(w)
    a = O.quantize(wb, bits)
    b = O.quantize(O.bf16_bits_to_f32(wb), bits)
    assert all(_same(x, y) for x, y in zip(a, b))


@pytest.mark.parametrize("bits", [4, 8])
def test_golden_reference_weight(golden, bits):
    w = O.reference_weight(256, 512)
    wq, s, b = O.quantize(w, bits)
    assert _same(wq, golden[f"ref_b{bits}_wq"])
    assert _same(s, golden[f"ref_b{bits}_scales"])
    assert _same(b, golden[f"ref_b{bits}_biases"])
    assert _same(O.dequantize(wq, s, b, 256, 512, bits), golden[f"ref_b{bits}_dequant"])
    y = O.qmatmul(O.f32_to_bf16_bits(O.reference_activation(8, 512)), wq, s, b, 256, bits)
    assert _same(y, golden[f"ref_b{bits}_qmm"])


@pytest.mark.parametrize("bits", [4, 8])
def test_golden_edge_cases(golden, bits):
    ew = golden["edge_w"]
    wq, s, b = O.quantize(ew, bits)
    assert _same(wq, golden[f"edge_b{bits}_wq"])
    assert _same(s, golden[f"edge_b{bits}_scales"])
    assert _same(b, golden[f"edge_b{bits}_biases"])
    assert _same(O.dequantize(wq, s, b, 8, 128, bits), golden[f"edge_b{bits}_dequant"])
    # NumPy agrees on every special group too.
    nq, ns, nb = O.np_quantize(ew, bits)
    assert _same(wq, nq) and _same(s, ns) and _same(b, nb)


def test_edge_case_semantics(golden):
    """The rules the header writes down, checked on the special groups."""
    s = O.bf16_bits_to_f32(golden["edge_b4_scales"])
    b = O.bf16_bits_to_f32(golden["edge_b4_biases"])
    d = O.bf16_bits_to_f32(golden["edge_b4_dequant"])
    # constant group: scale 0, every value reconstructs to bf16(0.25)
    assert s[0, 0] == 0 and (d[0, :64] == np.float32(0.25)).all()
    # +0/-0 group: bias is -0 (total order puts -0 below +0)
    assert b[1, 0] == 0 and np.signbit(b[1, 0])
    # exact integers 0..63 at 4 bits: scale 63/15 = 4.2 -> bf16, bias 0
    assert b[2, 0] == 0 and s[2, 0] == O.bf16_bits_to_f32(O.f32_to_bf16_bits(np.float32(63 / 15)))
    # a NaN member is ignored for the extrema
    assert np.isfinite(s[3, 0]) and b[3, 0] == np.float32(-2.0)
    # all-NaN group: +inf bias, and the dequantised values are NaN (canonical 0x7fff)
    assert np.isposinf(b[4, 0])
    assert (golden["edge_b4_dequant"][4, :64] == 0x7FFF).all()


def test_seeded_rng(golden):
    """SeededRng (lib.rs:104-145): deterministic, standard normal, pair order cos then sin."""
    assert _same(O.seeded_normals(0, 64), golden["rng_seed0_64"])
    assert _same(O.seeded_normals(42, 65), golden["rng_seed42_65"])
    # a prefix of a longer draw is the shorter draw
    assert _same(O.seeded_normals(42, 64), O.seeded_normals(42, 65)[:64])
    v = O.seeded_normals(5, 200_000).astype(np.float64)
    assert abs(v.mean()) < 0.01 and abs(v.std() - 1) < 0.01


# ------------------------------------------------ the reference's own thresholds

def test_round_trip_cost_is_what_the_bit_width_says():
    """mlx_quantized.rs:53-75: cosine > 0.99 for both widths, and 8-bit beats 4-bit."""
    w = O.reference_weight(256, 512)
    prev = 0.0
    for bits in (4, 8):
        wq, s, b = O.quantize(w, bits)
        back = O.bf16_bits_to_f32(O.dequantize(wq, s, b, 256, 512, bits))
        assert back.shape == w.shape
        c = O.cosine(w, back)
        assert c > 0.99, (bits, c)
        assert c > prev, (bits, c, prev)
        prev = c


def test_quantized_matmul_agrees_with_the_dense_one():
    """mlx_quantized.rs:83-117: X[8,512] @ W[256,512]^T, cosine > 0.999 against the dense
    f32 product, for 4 and 8 bits (the activation enters as bf16 here)."""
    w = O.reference_weight(256, 512)
    x = O.reference_activation(8, 512)
    want = x.astype(np.float64) @ w.astype(np.float64).T
    for bits in (4, 8):
        wq, s, b = O.quantize(w, bits)
        got = O.qmatmul(O.f32_to_bf16_bits(x), wq, s, b, 256, bits)
        assert got.shape == (8, 256)
        assert O.cosine(want, got) > 0.999, bits


def test_quantising_shrinks_the_weight_by_what_it_claims():
    """mlx_quantized.rs:120-141: resident/dense < 0.20 (4-bit), < 0.35 (8-bit) at 1024x1024,
    counting 4 bytes per scale and bias as mlx.rs:1981-1985 does."""
    dense = 1024 * 1024 * 4
    for bits, most in ((4, 0.20), (8, 0.35)):
        r = O.resident_bytes(1024, 1024, bits) / dense
        assert r < most, (bits, r)
    assert O.resident_bytes(1024, 1024, 4) == 1024 * 1024 // 2 + 2 * 1024 * 16 * 4


def test_oracle_rejects_what_the_reference_cannot_quantise():
    with pytest.raises(ValueError):
        O.quantize(np.zeros((4, 100), np.float32), 4)   # K % 64 != 0 stays dense
    with pytest.raises(ValueError):
        O.quantize(np.zeros((4, 64), np.float32), 3)


# ---------------------------------------------------------------- fused output stage

def test_epilogue_activations_match_torch_independent_implementations():
    """The oracle's gelu_approx / silu (restated from the reference's formulas) against torch's
    own CPU implementations in f64."""
    import torch
    a = np.linspace(-12.0, 12.0, 4001).reshape(1, -1)
    ta = torch.from_numpy(a)
    g = O.epilogue(a, act=O.ACT_GELU_TANH)
    s = O.epilogue(a, act=O.ACT_SILU)
    assert np.max(np.abs(g - torch.nn.functional.gelu(ta, approximate="tanh").numpy())) < 1e-12
    assert np.max(np.abs(s - torch.nn.functional.silu(ta).numpy())) < 1e-12
    assert np.array_equal(O.epilogue(a), a)


def test_epilogue_order_is_residual_plus_gate_times_activation_of_biased_product():
    acc = np.array([[1.0, -2.0], [0.5, 3.0]], np.float32)
    bias = O.f32_to_bf16_bits(np.array([0.5, 1.0], np.float32))
    gate = O.f32_to_bf16_bits(np.array([2.0, -1.0], np.float32))
    resid = O.f32_to_bf16_bits(np.array([[10.0, 20.0], [30.0, 40.0]], np.float32))
    y = O.epilogue(acc, bias, O.ACT_SILU, gate, resid)
    silu = lambda v: v / (1.0 + np.exp(-v))
    want = np.array([[10 + 2 * silu(1.5), 20 - silu(-1.0)], [30 + 2 * silu(1.0), 40 - silu(4.0)]])
    assert np.allclose(y, want, rtol=0, atol=1e-12)
