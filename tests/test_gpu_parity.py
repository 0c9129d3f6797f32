"""GPU parity: libsdq (through its C ABI) against the CPU oracle.

Bars (from the task's north star):
  * quantise (packed words, scales, biases) and dequantise: bit-exact;
  * quantised matmul: max|y - ref| / max|ref| <= 1e-2 and cosine >= 0.9999 against the
    f32 (f64-accumulated) dense product of the dequantised weights.
Full benchmark sizes are checked through sampled rows/columns and through a
size-independent property: with X = I (M = K) the product is exactly dequant(W)^T.
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


def dev_bf16(bits16: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits16).view(np.int16)).cuda().view(torch.bfloat16)


def host_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


def dev_u32(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).cuda()


def close(got_bf16: torch.Tensor, want: np.ndarray):
    g = got_bf16.float().cpu().numpy().astype(np.float64)
    w = want.astype(np.float64)
    rel = float(np.max(np.abs(g - w)) / max(np.max(np.abs(w)), 1e-30))
    cos = O.cosine(w, g)
    return rel, cos


def assert_close(got, want, what=""):
    rel, cos = close(got, want)
    assert rel <= MAX_ABS_REL and cos >= MIN_COSINE, f"{what}: max-abs-rel {rel:.3e}, cosine {cos:.7f}"


def quantize_both(w: np.ndarray, bits: int, wdtype=torch.float32):
    if wdtype == torch.float32:
        wd = torch.from_numpy(w).cuda()
        ref = O.quantize(w, bits)
    else:
        wb = O.f32_to_bf16_bits(w)
        wd = dev_bf16(wb)
        ref = O.quantize(wb, bits)
    got = sdq.quantize(wd, 64, bits)
    torch.cuda.synchronize()
    return got, ref


# ---------------------------------------------------------------- quantise / dequantise

@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("wdtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,k", [(256, 512), (1, 64), (3, 192), (129, 3072), (3072, 3072)])
def test_quantize_and_dequantize_bit_exact(bits, wdtype, n, k):
    w = O.seeded_normals(n * 7 + k, n * k).reshape(n, k) * np.float32(0.02)
    (wq, s, b), (rwq, rs, rb) = quantize_both(w, bits, wdtype)
    assert (wq.cpu().numpy().view(np.uint32) == rwq).all(), "packed words"
    assert (host_bits(s) == rs).all(), "scales"
    assert (host_bits(b) == rb).all(), "biases"
    d = sdq.dequantize(wq, s, b, 64, bits)
    want = O.dequantize(rwq, rs, rb, n, k, bits)
    assert (host_bits(d) == want).all(), "dequant bf16"
    d32 = sdq.dequantize(wq, s, b, 64, bits, out_dtype=torch.float32).cpu().numpy()
    assert (d32.view(np.uint32) == (want.astype(np.uint32) << 16)).all(), "dequant f32"


@pytest.mark.parametrize("bits", [4, 8])
def test_edge_cases_bit_exact(bits):
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "quantized_linear.npz"))
    ew = g["edge_w"]
    wq, s, b = sdq.quantize(torch.from_numpy(ew).cuda(), 64, bits)
    assert (wq.cpu().numpy().view(np.uint32) == g[f"edge_b{bits}_wq"]).all()
    assert (host_bits(s) == g[f"edge_b{bits}_scales"]).all()
    assert (host_bits(b) == g[f"edge_b{bits}_biases"]).all()
    assert (host_bits(sdq.dequantize(wq, s, b, 64, bits)) == g[f"edge_b{bits}_dequant"]).all()


@pytest.mark.parametrize("bits", [4, 8])
def test_reference_weight_matches_golden(bits):
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "quantized_linear.npz"))
    w = O.reference_weight(256, 512)
    wq, s, b = sdq.quantize(torch.from_numpy(w).cuda(), 64, bits)
    assert (wq.cpu().numpy().view(np.uint32) == g[f"ref_b{bits}_wq"]).all()
    x = dev_bf16(O.f32_to_bf16_bits(O.reference_activation(8, 512)))
    y = sdq.quantized_matmul(x, wq, s, b, 64, bits)
    assert_close(y, g[f"ref_b{bits}_qmm"], f"golden qmm {bits}")


# ---------------------------------------------------------------- quantised matmul

def run_qmm(m, k, n, bits, seed, with_bias=False, sigma_w=0.02):
    xb, w = O.synthetic_linear(seed, m, k, n, sigma_w)
    rwq, rs, rb = O.quantize(w, bits)
    bias = None
    if with_bias:
        bias = O.f32_to_bf16_bits(O.seeded_normals(seed + 1, n) * np.float32(0.5))
    y = sdq.quantized_matmul(dev_bf16(xb), dev_u32(rwq), dev_bf16(rs), dev_bf16(rb), 64, bits,
                             bias=None if bias is None else dev_bf16(bias))
    sdq.device_status()
    want = O.qmatmul(xb, rwq, rs, rb, n, bits, bias)
    return y, want


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 7, 8])
@pytest.mark.parametrize("k,n", [(64, 16), (128, 40), (3072, 256), (640, 1000)])
def test_small_m(bits, m, k, n):
    y, want = run_qmm(m, k, n, bits, seed=m * 100 + n)
    assert y.shape == (m, n)
    assert_close(y, want, f"small-M m={m} k={k} n={n} bits={bits}")


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m", [9, 16, 64, 65, 128, 129, 256, 300, 1024])
@pytest.mark.parametrize("k,n", [(64, 128), (192, 200), (3072, 384)])
def test_large_m(bits, m, k, n):
    y, want = run_qmm(m, k, n, bits, seed=m * 1000 + k + n)
    assert y.shape == (m, n)
    assert_close(y, want, f"large-M m={m} k={k} n={n} bits={bits}")


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m", [1, 3, 8])
@pytest.mark.parametrize("k,n", [(256, 1), (256, 37), (512, 203), (3072, 2048), (3072, 4096),
                                 (3072, 9216), (1024, 18432)])
def test_small_m_weight_stream(bits, m, k, n):
    """M <= 8 with K a whole number of 128-byte weight rows: the streaming kernel, at each of its
    tile heights (N = 2048 / 4096 / 9216 / 18432 pick 16 / 32 / 64 / 128 rows) and ragged N."""
    y, want = run_qmm(m, k, n, bits, seed=31 * m + k + n, with_bias=(n % 2 == 1))
    assert y.shape == (m, n)
    assert_close(y, want, f"stream m={m} k={k} n={n} bits={bits}")


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m", [3, 130, 300])
@pytest.mark.parametrize("n", [1, 37, 203])
def test_output_width_not_a_multiple_of_8(bits, m, n):
    """Rows of Y that are not 16-byte multiples are written with plain stores, not TMA."""
    y, want = run_qmm(m, 192, n, bits, seed=17 + m + n, with_bias=True)
    assert_close(y, want, f"odd n={n} m={m} bits={bits}")


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m", [4, 300])
def test_fused_bias(bits, m):
    y, want = run_qmm(m, 256, 192, bits, seed=5 + m, with_bias=True)
    assert_close(y, want, f"bias m={m} bits={bits}")


@pytest.mark.parametrize("m,k,bits", [(4, 16384, 4), (8, 12288, 8), (3, 12288, 8), (8, 64, 8),
                                       (6, 192, 4), (8, 25600, 4)])
def test_small_m_long_k(m, k, bits):
    """Long K at small M: staged in shared memory when it fits, else the tensor-core path."""
    y, want = run_qmm(m, k, 160, bits, seed=11 + m + k)
    assert_close(y, want, f"m={m} k={k} bits={bits}")


@pytest.mark.parametrize("bits,k,n", [(4, 3072, 18432), (8, 12288, 3072),
                                      (4, 1024, 3072), (4, 4096, 3072), (8, 1024, 3072)])
def test_identity_activation_reproduces_the_dequantised_weight(bits, k, n):
    """Full-size property: X = I (M = K) gives Y = dequant(W)^T exactly, since each output is
    one exact product; checks the tensor-core path against the dequantise kernel bit for bit.
    M = 1024 and 4096 against N = 3072 select the 176- and 240-token tiles."""
    w = torch.randn(n, k, device="cuda", generator=torch.Generator("cuda").manual_seed(bits)) * 0.02
    wq, s, b = sdq.quantize(w, 64, bits)
    eye = torch.eye(k, device="cuda", dtype=torch.bfloat16)
    y = sdq.quantized_matmul(eye, wq, s, b, 64, bits)
    d = sdq.dequantize(wq, s, b, 64, bits)
    sdq.device_status()
    assert torch.equal(y.view(torch.int16), d.t().contiguous().view(torch.int16))


@pytest.mark.parametrize("bits,k,n", [(4, 3072, 1000), (8, 3072, 1000), (4, 4096, 384), (8, 1024, 200)])
def test_identity_rows_at_sixteen_tokens(bits, k, n):
    """M = 16 runs the tensor-core kernel with X resident (K = 1024, 3072 and 4096; W4 and W8;
    N not a multiple of the 128-feature tile).  Sixteen rows of the identity pick sixteen
    columns of dequant(W)^T, each output one exact product; the windows cover every k, so the
    A operand of every step is checked against the dequantise kernel bit for bit."""
    w = torch.randn(n, k, device="cuda", generator=torch.Generator("cuda").manual_seed(k + bits)) * 0.02
    wq, s, b = sdq.quantize(w, 64, bits)
    d = sdq.dequantize(wq, s, b, 64, bits)
    eye = torch.eye(k, device="cuda", dtype=torch.bfloat16)
    for j0 in range(0, k, 16):
        y = sdq.quantized_matmul(eye[j0:j0 + 16], wq, s, b, 64, bits)
        if not torch.equal(y.view(torch.int16), d[:, j0:j0 + 16].t().contiguous().view(torch.int16)):
            raise AssertionError(f"k window {j0}..{j0 + 15} differs from the dequantised weight")
    sdq.device_status()


@pytest.mark.parametrize("m", [1, 2, 4, 8])
def test_config3_full_size_every_m(m):
    """Benchmark configuration 3 at full size and at every M it names: X [M, 3072] against the
    whole [18432, 3072] W4 weight (the adaLN modulation shape), every output checked against the
    oracle's f64 product of the dequantised weights, on the SeededRng draw of the benchmark."""
    k, n, bits = 3072, 18432, 4
    xb, w = O.synthetic_linear(300 + m, m, k, n, 0.02)
    rwq, rs, rb = O.quantize(w, bits)
    y = sdq.quantized_matmul(dev_bf16(xb), dev_u32(rwq), dev_bf16(rs), dev_bf16(rb), 64, bits)
    sdq.device_status()
    assert y.shape == (m, n)
    want = O.qmatmul(xb, rwq, rs, rb, n, bits)
    assert_close(y, want, f"config 3 m={m}")


@pytest.mark.parametrize("cfg", ["c1", "c2", "c3", "c5"])
def test_baseline_configs_sampled(cfg):
    """The benchmark configurations at full size; the oracle checks a sample of rows and columns."""
    shapes = {"c1": (1024, 3072, 3072, 4, 0.02), "c2": (4096, 12288, 3072, 8, 0.01),
              "c3": (8, 3072, 18432, 4, 0.02), "c5": (16384, 3072, 12288, 4, 0.02)}
    m, k, n, bits, sig = shapes[cfg]
    gen = torch.Generator("cuda").manual_seed(hash(cfg) % 1000)
    x = torch.randn(m, k, device="cuda", generator=gen).to(torch.bfloat16)
    w = torch.randn(n, k, device="cuda", generator=gen) * sig
    wq, s, b = sdq.quantize(w, 64, bits)
    y = sdq.quantized_matmul(x, wq, s, b, 64, bits)
    sdq.device_status()
    rng = np.random.default_rng(0)
    im = np.sort(rng.choice(m, size=min(m, 96), replace=False))
    jn = np.sort(rng.choice(n, size=min(n, 256), replace=False))
    xs = host_bits(x[torch.from_numpy(im).cuda()])
    want = O.qmatmul(xs, wq[torch.from_numpy(jn).cuda()].cpu().numpy().view(np.uint32),
                     host_bits(s[torch.from_numpy(jn).cuda()]), host_bits(b[torch.from_numpy(jn).cuda()]),
                     len(jn), bits)
    got = y[torch.from_numpy(im).cuda()][:, torch.from_numpy(jn).cuda()]
    assert_close(got, want, cfg)


def test_device_status_is_clean_after_the_suite():
    sdq.device_status()


def test_misaligned_device_pointer_is_rejected():
    x = torch.zeros(4 * 128 + 8, device="cuda", dtype=torch.bfloat16)[1:1 + 4 * 128].view(4, 128)
    wq, s, b = sdq.quantize(torch.zeros(64, 128, device="cuda"), 64, 4)
    with pytest.raises(sdq.SdqError) as e:
        sdq.quantized_matmul(x, wq, s, b, 64, 4)
    assert e.value.code == sdq.SDQ_ERR_INVALID
