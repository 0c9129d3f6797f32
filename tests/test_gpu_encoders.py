"""The quantised linear at its other consumers' shapes (sdq.encoders): text-encoder layers
(T5-XXL, Qwen3-4B, Qwen2.5-VL-7B, Mistral Small 3.2) at 256 and 512 prompt tokens, and Flux's
M = 1 conditioning MLPs.  The kernel runs at the full shape; rows of the output -- the first
and last of the activation and rows on either side of token-tile boundaries -- are checked
against the oracle (f64 product of the dequantised weight), with the matmul's bars."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
import sdq
from sdq import encoders as E
from conftest import gpu_available

MAX_ABS_REL = 1e-2
MIN_COSINE = 0.9999


def _unique(table):
    seen, out = set(), []
    for name, n, k, m in table:
        if (n, k, m) not in seen:
            seen.add((n, k, m))
            out.append((name, n, k, m))
    return out


ENCODER_CASES = _unique([lin for e in E.ENCODERS for t in (256, 512) for lin in E.layer_linears(e, t)])
CONDITIONING_CASES = _unique(E.flux_conditioning())


def test_tables_follow_the_reference_configurations():
    t5 = E.layer_linears(E.T5_XXL, 512)
    assert [(n, k) for _, n, k, _ in t5] == [(4096, 4096)] * 4 + [(10240, 4096)] * 2 + [(4096, 10240)]
    mistral = E.layer_linears(E.MISTRAL_SMALL_3_2, 256)
    assert [(n, k) for _, n, k, _ in mistral] == [(4096, 5120), (1024, 5120), (1024, 5120), (5120, 4096),
                                                  (32768, 5120), (32768, 5120), (5120, 32768)]
    assert all(k % 64 == 0 for _, _, k, _ in ENCODER_CASES + CONDITIONING_CASES)
    assert len(E.flux_conditioning()) == 7 and len(CONDITIONING_CASES) == 4
    assert all(m == 1 for *_, m in CONDITIONING_CASES)


def _rows(m):
    rows = {0, 1, m - 2, m - 1}
    for edge in (16, 64, 128, 176, 240, 256):
        if edge < m:
            rows |= {edge - 1, edge}
    return sorted(r for r in rows if 0 <= r < m)


@pytest.mark.gpu
@pytest.mark.skipif(not gpu_available(), reason="needs an sm_100 device")
@pytest.mark.parametrize("name,n,k,m", ENCODER_CASES + CONDITIONING_CASES,
                         ids=[f"{n}x{k}@{m}" for _, n, k, m in ENCODER_CASES + CONDITIONING_CASES])
def test_consumer_shape_matches_the_oracle(name, n, k, m):
    bits = 8 if n * k <= 4096 * 4096 else 4        # both widths across the table
    g = torch.Generator("cuda").manual_seed(n + 7 * k + m)
    w = torch.randn(n, k, device="cuda", generator=g) * 0.02
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    wq, s, b = sdq.quantize(w, 64, bits)
    del w
    y = sdq.quantized_matmul(x, wq, s, b, 64, bits)
    sdq.device_status()
    rows = _rows(m)
    xs = x[rows].contiguous().cpu().view(torch.int16).numpy().view(np.uint16)
    want = O.qmatmul(xs, wq.cpu().numpy().view(np.uint32), s.cpu().view(torch.int16).numpy().view(np.uint16),
                     b.cpu().view(torch.int16).numpy().view(np.uint16), n, bits).astype(np.float64)
    got = y[rows].float().cpu().numpy().astype(np.float64)
    rel = float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))
    cos = O.cosine(want, got)
    assert rel <= MAX_ABS_REL and cos >= MIN_COSINE, f"{name} W{bits}: max-abs-rel {rel:.3e}, cosine {cos:.7f}"
