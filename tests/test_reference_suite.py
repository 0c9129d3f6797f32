"""The reference's own quantised-weight tests, restated against libsdq on the GPU.

Each test mirrors one in crates/sd-models/tests/mlx_quantized.rs (same deterministic
inputs, same assertions), with MLX replaced by the C ABI.  The dense reference products
are computed in f64 on the host."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
import sdq
from conftest import gpu_available
from sdq import quantized as Q

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not gpu_available(), reason="needs an sm_100 device")]


def weight(out, inp):
    return torch.from_numpy(O.reference_weight(out, inp)).cuda()


def activation(rows, inp):
    return torch.from_numpy(O.reference_activation(rows, inp)).cuda()


def test_the_round_trip_cost_is_what_the_bit_width_says():
    """mlx_quantized.rs:53-75."""
    w = weight(256, 512)
    previous = 0.0
    for bits in (4, 8):
        q = sdq.QuantizedArray.quantize(w, Q.GROUP_SIZE, bits)
        back = q.dequantize(out_dtype=torch.float32)
        assert tuple(back.shape) == tuple(w.shape)
        c = O.cosine(w.cpu().numpy(), back.cpu().numpy())
        assert c > 0.99, f"{bits}-bit lost too much: cosine {c:.6f}"
        assert c > previous, "8-bit is no better than 4-bit"
        previous = c


def test_the_quantized_matmul_agrees_with_the_dense_one():
    """mlx_quantized.rs:83-117 (activations enter as bf16, the library's input type)."""
    out, inp = 256, 512
    w = weight(out, inp)
    x = activation(8, inp)
    want = x.double().cpu().numpy() @ w.double().cpu().numpy().T
    for bits in (4, 8):
        q = sdq.QuantizedArray.quantize(w, Q.GROUP_SIZE, bits)
        got = q.matmul(x.to(torch.bfloat16))
        assert tuple(got.shape) == (8, out)
        c = O.cosine(want, got.float().cpu().numpy())
        assert c > 0.999, f"{bits}-bit matmul correlates only {c:.6f}"


def test_quantising_shrinks_the_weight_by_what_it_claims():
    """mlx_quantized.rs:120-141."""
    out, inp = 1024, 1024
    w = weight(out, inp)
    dense_bytes = out * inp * 4
    for bits, most in ((4, 0.20), (8, 0.35)):
        q = sdq.QuantizedArray.quantize(w, Q.GROUP_SIZE, bits)
        ratio = q.resident_bytes() / dense_bytes
        assert ratio < most, f"{bits}-bit came to {ratio * 100:.1f}% of dense"
        assert q.resident_bytes() == sdq.resident_bytes(out, inp, bits)


def test_the_split_leaves_norms_and_odd_widths_dense():
    """mlx_quantized.rs:148-179."""
    w = {
        "blk.0.attn.weight": weight(128, 256),
        "blk.0.attn.bias": torch.zeros(128, device="cuda"),
        "blk.0.norm.weight": torch.ones(128, device="cuda"),
        "blk.0.odd.weight": weight(32, 100),
    }
    q = Q.from_dense(w, Q.DEFAULT_BITS)
    assert "blk.0.attn.weight" in q.quantized
    assert "blk.0.attn.bias" in q.dense
    assert "blk.0.norm.weight" in q.dense
    assert "blk.0.odd.weight" in q.dense
    assert len(q) == 4
    for name in w:
        assert q.contains_key(name)


def test_the_linear_dispatches_to_the_right_kernel():
    """mlx_quantized.rs:182-228."""
    dense_map = {"big.weight": weight(128, 256), "small.weight": weight(8, 32)}
    x_big = activation(4, 256)
    x_small = activation(4, 32)
    want_big = x_big.double() @ dense_map["big.weight"].double().t()
    want_small = x_small @ dense_map["small.weight"].t()
    q = Q.from_dense(dense_map, 8)
    assert "big.weight" in q.quantized
    assert "small.weight" in q.dense
    got_big = Q.linear(x_big.to(torch.bfloat16), "big.weight", None, q)
    c = O.cosine(want_big.cpu().numpy(), got_big.float().cpu().numpy())
    assert c > 0.999
    got_small = Q.linear(x_small, "small.weight", None, q)
    worst = (want_small - got_small).abs().max().item()
    assert worst < 1e-5, "the dense branch is not the dense matmul"
    with pytest.raises(sdq.SdqError):
        Q.linear(x_big, "absent.weight", None, q)
    with pytest.raises(sdq.SdqError):
        q.dense_tensor("big.weight")   # quantised: reach it through linear
