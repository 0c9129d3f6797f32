"""The load-time pipeline from GGUF (sdq.gguf, sdq_gguf_quantize / sdq_gguf_dequantize,
sdq.quantized.from_gguf): the reader against the writer and against gguf-py, the oracle's block
decoders against the reference's own known answers and against gguf-py (llama.cpp's
implementation, version 0.19.0 in this image), and on a GPU the kernels bit for bit against
the oracle."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from sdq import gguf as G
from sdq._abi import SDQ_ERR_INVALID, SDQ_ERR_UNSUPPORTED, SdqError
from conftest import gpu_available

F16_FIELDS = {G.Q4_0: [0], G.Q8_0: [0], G.Q4_K: [0, 2], G.Q5_K: [0, 2], G.Q6_K: [208]}
BLOCK_TYPES = [G.Q4_0, G.Q8_0, G.Q4_K, G.Q5_K, G.Q6_K]
ALL_TYPES = [G.F32, G.F16, G.BF16] + BLOCK_TYPES


def random_raw(kind: int, count: int, seed: int) -> np.ndarray:
    """Valid block bytes for `count` values: random bytes, with every f16 scale field a finite
    half (blocks of GGUF files hold finite scales)."""
    rng = np.random.default_rng(seed)
    per, nb = G.BLOCKS[kind]
    if per == 1:
        v = (rng.standard_normal(count) * 0.05).astype(np.float32)
        if kind == G.F32:
            return v.view(np.uint8).copy()
        if kind == G.F16:
            return v.astype(np.float16).view(np.uint8).copy()
        return (v.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8).copy()
    blocks = count // per
    raw = rng.integers(0, 256, size=(blocks, nb), dtype=np.uint8)
    for off in F16_FIELDS[kind]:
        raw[:, off:off + 2] = (rng.standard_normal(blocks) * 0.01).astype(np.float16).view(np.uint8).reshape(blocks, 2)
    return raw.reshape(-1)


# ---------------------------------------------------------------- oracle known answers

def _half_by_exponent(h: int) -> float:
    """The reference's independent conversion (mlx_gguf.rs:472-488): exponent arithmetic."""
    sign, exp, frac = (h >> 15) & 1, (h >> 10) & 0x1F, h & 0x3FF
    if exp == 0:
        v = frac * 2.0 ** -24
        return -v if sign else v
    if exp == 0x1F:
        return np.uint32((sign << 31) | (0xFF << 23) | (frac << 13)).view(np.float32)
    return np.uint32((sign << 31) | ((exp + 112) << 23) | (frac << 13)).view(np.float32)


def test_f16_decode_is_exact_for_every_bit_pattern():
    """mlx_gguf.rs:455-470: all 65536 half patterns against the exponent-arithmetic form."""
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = O.gguf_dequantize(bits.view(np.uint8), O.GGML_F16, 65536)
    want = np.array([_half_by_exponent(int(h)) for h in bits], dtype=np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def test_bf16_is_f32s_top_half_and_not_f16():
    """mlx_gguf.rs:492-544: widening is a shift; 0x3f80 is 1.0 and 0x4900 is 524288."""
    raw = np.array([0x3F80, 0x4900, 0x8000, 0x7F80, 0x7FC0], np.uint16).view(np.uint8)
    v = O.gguf_dequantize(raw, O.GGML_BF16, 5)
    assert v[0] == 1.0 and v[1] == 524288.0 and v[2] == 0.0 and np.signbit(v[2])
    assert np.isinf(v[3]) and np.isnan(v[4])


def test_oracle_block_decoders_match_gguf_py():
    quants = pytest.importorskip("gguf.quants")
    from gguf import GGMLQuantizationType as T
    types = {G.Q4_0: T.Q4_0, G.Q8_0: T.Q8_0, G.Q4_K: T.Q4_K, G.Q5_K: T.Q5_K, G.Q6_K: T.Q6_K}
    for kind, t in types.items():
        raw = random_raw(kind, 64 * 256, seed=kind)
        ours = O.gguf_dequantize(raw, kind, 64 * 256)
        theirs = quants.dequantize(raw.reshape(1, -1), t).reshape(-1).astype(np.float32)
        assert np.array_equal(ours.view(np.uint32), theirs.view(np.uint32)), G.NAMES[kind]


# ---------------------------------------------------------------- reader / writer

def _sample_file(path, alignment=32):
    specs = [("blk.0.attn_q.weight", (256, 512), G.Q4_K), ("token_embd.weight", (64, 256), G.Q8_0),
             ("blk.0.ffn_down.weight", (512, 256), G.Q6_K), ("norm.weight", (512,), G.F32),
             ("blk.0.attn_k.weight", (128, 256), G.Q5_K), ("blk.0.attn_v.weight", (64, 96), G.Q4_0),
             ("out.weight", (32, 64), G.BF16), ("pos.weight", (2, 3, 64), G.F16)]
    tensors = [(n, s, k, random_raw(k, int(np.prod(s)), seed=i)) for i, (n, s, k) in enumerate(specs)]
    G.write(str(path), tensors, metadata={"demo.count": 7}, alignment=alignment)
    return tensors


@pytest.mark.parametrize("alignment", [32, 64])
def test_reader_reads_back_what_the_writer_wrote(tmp_path, alignment):
    tensors = _sample_file(tmp_path / "m.gguf", alignment)
    g = G.Gguf(str(tmp_path / "m.gguf"))
    assert g.alignment == alignment and g.data_start % alignment == 0
    assert [(t.name, t.shape, t.kind) for t in g.tensors] == [(n, tuple(s), k) for n, s, k, _ in tensors]
    for info, (_, _, _, raw) in zip(g.tensors, tensors):
        assert np.array_equal(g.raw(info), raw)


def test_gguf_py_reads_the_written_file(tmp_path):
    gguf = pytest.importorskip("gguf")
    tensors = _sample_file(tmp_path / "m.gguf")
    r = gguf.GGUFReader(str(tmp_path / "m.gguf"))
    assert [t.name for t in r.tensors] == [n for n, *_ in tensors]
    for t, (_, shape, kind, raw) in zip(r.tensors, tensors):
        assert int(t.tensor_type) == kind
        assert tuple(int(d) for d in reversed(t.shape)) == tuple(shape)
        assert np.array_equal(np.asarray(t.data).view(np.uint8).reshape(-1), raw)


def test_reader_rejects_what_the_reference_rejects(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGML" + b"\0" * 60)
    with pytest.raises(SdqError) as e:
        G.Gguf(str(p))
    assert e.value.code == SDQ_ERR_INVALID and "not a GGUF file" in str(e.value)
    G.write(str(p), [("w", (4, 32), 3, np.zeros(4 * 20, np.uint8))])     # type 3 = Q4_1
    with pytest.raises(SdqError) as e:
        G.Gguf(str(p))
    assert e.value.code == SDQ_ERR_UNSUPPORTED and "Q4_K" in str(e.value)
    data = bytearray(p.read_bytes())
    data[4:8] = (1).to_bytes(4, "little")
    p.write_bytes(bytes(data))
    with pytest.raises(SdqError) as e:
        G.Gguf(str(p))
    assert e.value.code == SDQ_ERR_UNSUPPORTED and "version 1" in str(e.value)


# ---------------------------------------------------------------- GPU kernels

def _dev(raw):
    import torch
    return torch.from_numpy(raw.copy()).cuda()


@pytest.mark.gpu
@pytest.mark.skipif(not gpu_available(), reason="needs an sm_100 device")
@pytest.mark.parametrize("kind", ALL_TYPES, ids=[G.NAMES[k] for k in ALL_TYPES])
def test_gpu_dequantize_is_the_reference_f32_bit_for_bit(kind):
    import sdq
    import torch
    shape = (96, 512)
    raw = random_raw(kind, shape[0] * shape[1], seed=100 + kind)
    want = O.gguf_dequantize(raw, kind, shape[0] * shape[1]).reshape(shape)
    got = sdq.gguf_dequantize(_dev(raw), kind, shape).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    got16 = sdq.gguf_dequantize(_dev(raw), kind, shape, torch.bfloat16).cpu().view(torch.int16).numpy()
    assert np.array_equal(got16.view(np.uint16), O.f32_to_bf16_bits(want))



@pytest.mark.gpu
@pytest.mark.skipif(not gpu_available(), reason="needs an sm_100 device")
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("kind", ALL_TYPES, ids=[G.NAMES[k] for k in ALL_TYPES])
def test_gpu_quantize_from_blocks_equals_quantising_the_dequantised_tensor(kind, bits):
    import sdq
    import torch
    n, k = 80, 768
    raw = random_raw(kind, n * k, seed=200 + kind)
    dense = O.gguf_dequantize(raw, kind, n * k).reshape(n, k)
    wq, s, b = sdq.gguf_quantize(_dev(raw), kind, n, k, bits)
    rwq, rs, rb = sdq.quantize(torch.from_numpy(dense).cuda(), 64, bits)
    sdq.device_status()
    assert torch.equal(wq, rwq) and torch.equal(s.view(torch.int16), rs.view(torch.int16))
    assert torch.equal(b.view(torch.int16), rb.view(torch.int16))
    owq, os_, ob = O.quantize(dense, bits)               # and the CPU oracle, from the same values
    assert np.array_equal(wq.cpu().numpy().view(np.uint32), owq)
    assert np.array_equal(s.cpu().view(torch.int16).numpy().view(np.uint16), os_)
    assert np.array_equal(b.cpu().view(torch.int16).numpy().view(np.uint16), ob)


@pytest.mark.gpu
@pytest.mark.skipif(not gpu_available(), reason="needs an sm_100 device")
def test_from_gguf_quantises_by_the_reference_policy(tmp_path):
    import sdq
    import torch
    from sdq import quantized as Q
    specs = [("double_blocks.0.img_attn.qkv.weight", (384, 256), G.Q4_K),     # 4 bits
             ("img_in.weight", (256, 64), G.Q8_0),                           # sensitive: 8 bits
             ("double_blocks.0.img_mlp.2.weight", (256, 512), G.Q6_K),        # 4 bits
             ("double_blocks.0.img_attn.norm.query_norm.scale", (128,), G.F32),  # 1-D: dense
             ("x_embedder.proj.weight", (64, 256), G.BF16),                   # indexed: dense
             ("single_blocks.0.linear2.weight", (128, 512), G.Q5_K)]          # 4 bits
    tensors = [(n, s, k, random_raw(k, int(np.prod(s)), seed=300 + i)) for i, (n, s, k) in enumerate(specs)]
    path = str(tmp_path / "flux.gguf")
    G.write(path, tensors)
    w = Q.from_gguf(path, 4)
    assert sorted(w.quantized) == sorted(n for n, s, _ in specs if len(s) == 2 and n != "x_embedder.proj.weight")
    assert sorted(w.dense) == ["double_blocks.0.img_attn.norm.query_norm.scale", "x_embedder.proj.weight"]
    assert w.quantized["img_in.weight"].bits == 8 and w.quantized["double_blocks.0.img_attn.qkv.weight"].bits == 4
    for name, shape, kind, raw in tensors:
        dense = O.gguf_dequantize(raw, kind, int(np.prod(shape))).reshape(shape)
        if name in w.dense:
            got = w.dense[name].cpu().numpy()
            assert got.dtype == np.float32 and np.array_equal(got.view(np.uint32), dense.view(np.uint32))
        else:
            q = w.quantized[name]
            rwq, rs, rb = sdq.quantize(torch.from_numpy(dense).cuda(), 64, q.bits)
            assert torch.equal(q.weight, rwq) and torch.equal(q.scales.view(torch.int16), rs.view(torch.int16))
    # the loaded weights serve the linear as any quantised weight does
    x = torch.randn(5, 256, device="cuda").to(torch.bfloat16)
    y = w.linear(x, "double_blocks.0.img_attn.qkv.weight")
    q = w.quantized["double_blocks.0.img_attn.qkv.weight"]
    ref = x.float() @ sdq.dequantize(q.weight, q.scales, q.biases, 64, 4, torch.float32).t()
    assert float((y.float() - ref).abs().max() / ref.abs().max()) <= 1e-2
    dropped = Q.from_gguf_renamed(path, 4, lambda n: n if n.startswith("img_in") else None)
    assert list(dropped.quantized) == ["img_in.weight"] and not dropped.dense
    with pytest.raises(SdqError) as e:
        Q.from_gguf_renamed(path, 4, lambda n: None)
    assert "carries no tensors this model recognises" in str(e.value)


# ---------------------------------------------------------------- the synthetic-input draw

@pytest.mark.gpu
@pytest.mark.skipif(not gpu_available(), reason="needs an sm_100 device")
@pytest.mark.parametrize("seed,count", [(0, 1), (7, 1001), (2, 1 << 20)])
def test_gpu_seeded_normals_are_the_reference_draw(seed, count):
    """sdq_seeded_normals against the oracle's SeededRng (lib.rs:104-145).  The f64 log / sincos
    of the device and of the host libm may differ in the last f64 place, which moves an f32
    result by one unit in the rare case it lands on a rounding boundary."""
    import sdq
    got = sdq.seeded_normals(seed, count).cpu().numpy()
    want = O.seeded_normals(seed, count)
    diff = np.abs(got.view(np.int32).astype(np.int64) - want.view(np.int32).astype(np.int64))
    assert diff.max() <= 1 and np.count_nonzero(diff) <= max(1, count // 100000)
