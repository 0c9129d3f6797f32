"""The Flux-shaped stack built on the library (sdq.flux): its table of linears on CPU, and on a
GPU a small stack whose quantised forward is compared with the same forward run on a dense
source holding the dequantised weights (torch matmuls) -- the wiring of every linear, its bias
and its bit width, checked end to end."""
from __future__ import annotations

import pytest
import torch

from sdq import flux
from sdq.quantized import DenseWeights
from conftest import gpu_available


def test_whole_model_table_matches_the_configuration():
    cfg = flux.FluxShape()
    table = flux.linear_table(cfg)
    assert len(table) == 312
    assert abs(flux.flops(cfg) - 59.51e12) / 59.51e12 < 1e-3
    eight = [n for n, *_ in table if flux.bits_for(n) == 8]
    # out-projection and MLP down-projection of both streams in 19 double blocks, linear2 of 38 singles
    assert len(eight) == 19 * 4 + 38
    assert all(k % 64 == 0 for _, _, k, _ in table)
    packed = sum(n * k * flux.bits_for(name) / 8 + 4 * n * k / 64 for name, n, k, _ in table)
    assert 8.3e9 < packed < 8.6e9            # ~8.48 GB of packed weights, scales and biases


@pytest.mark.gpu
@pytest.mark.skipif(not gpu_available(), reason="needs an sm_100 device")
def test_small_stack_quantised_forward_matches_the_dense_forward():
    cfg = flux.FluxShape(hidden=256, heads=2, depth=2, depth_single=2, txt_tokens=32, img_tokens=64,
                         context_dim=128, vec_dim=64)
    qw, dense = flux.random_weights(cfg, seed=3, keep_dense=True)
    rope = flux.rope_tables(cfg)
    args = flux.inputs(cfg, seed=4)
    got = flux.forward(qw, *args, cfg, rope)
    want = flux.forward(DenseWeights(dense), *args, cfg, rope)
    torch.cuda.synchronize()
    assert got.shape == (1, cfg.img_tokens, cfg.in_channels)
    g, w = got.double().flatten(), want.double().flatten()
    cos = float(g @ w / (g.norm() * w.norm()))
    rel = float((g - w).abs().max() / w.abs().max())
    assert cos >= 0.999 and rel <= 5e-2, (cos, rel)


@pytest.mark.gpu
@pytest.mark.skipif(not gpu_available(), reason="needs an sm_100 device")
def test_fused_output_stages_match_the_op_by_op_forward():
    """The forward with gate / residual / activation fused into the linears against the same
    quantised weights with those ops run one by one after each linear."""
    from sdq.quantized import OpByOp
    cfg = flux.FluxShape(hidden=256, heads=2, depth=2, depth_single=2, txt_tokens=32, img_tokens=64,
                         context_dim=128, vec_dim=64)
    qw = flux.random_weights(cfg, seed=5)
    rope = flux.rope_tables(cfg)
    args = flux.inputs(cfg, seed=6)
    got = flux.forward(qw, *args, cfg, rope)
    want = flux.forward(OpByOp(qw), *args, cfg, rope)
    torch.cuda.synchronize()
    g, w = got.double().flatten(), want.double().flatten()
    cos = float(g @ w / (g.norm() * w.norm()))
    rel = float((g - w).abs().max() / w.abs().max())
    assert cos >= 0.999 and rel <= 5e-2, (cos, rel)
