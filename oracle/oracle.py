"""CPU oracle for the affine group-wise quantiser -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this module, and only as
the checker or the timed CPU baseline.  The product (``libsdq.so`` and the
``sdq`` package) never imports it and has no CPU fallback.

Two restatements of the same rule live here:

* ``liboracle`` -- ``oracle/sdq_oracle.c`` through ctypes (fast, OpenMP),
* ``np_*``      -- a NumPy restatement written independently from the C one,
  used to cross-check the C code bit for bit on small inputs.

Both follow the reference's seam: ``QuantizedArray::{quantize, dequantize,
matmul, resident_bytes}`` (crates/sd-tensor/src/mlx.rs:1846-1986), group 64 and
the K % 64 rule (crates/sd-models/src/mlx/quantized.rs:45-49, 168-174), and the
``SeededRng`` draw (crates/sd-tensor/src/lib.rs:104-145).  The arithmetic of
the reference lives in MLX (external, version unpinned, absent here): bit-level
parity with MLX is UNPINNED; the rounding rules written in ``sdq_oracle.h``
define the bits, and the reference's own test thresholds
(crates/sd-models/tests/mlx_quantized.rs:53-228) pin the behaviour.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsdq_oracle.so")
GROUP = 64

_lib = None


def build(force: bool = False) -> str:
    """Compile ``sdq_oracle.c`` into ``oracle/libsdq_oracle.so`` (gcc, OpenMP)."""
    if force or not os.path.exists(LIB_PATH) or (
        os.path.getmtime(LIB_PATH) < max(os.path.getmtime(os.path.join(HERE, f))
                                         for f in ("sdq_oracle.c", "sdq_oracle.h"))):
        subprocess.check_call(["make", "-s", "-C", HERE])
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        p, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.oracle_quantize_f32.argtypes = [p, i64, i64, i32, p, p, p]
        L.oracle_quantize_bf16.argtypes = [p, i64, i64, i32, p, p, p]
        L.oracle_dequantize_bf16.argtypes = [p, p, p, i64, i64, i32, p]
        L.oracle_qmatmul.argtypes = [p, i64, i64, p, p, p, i64, i32, p, p, i32]
        L.oracle_resident_bytes.argtypes = [i64, i64, i32, i32]
        L.oracle_resident_bytes.restype = ctypes.c_size_t
        L.oracle_seeded_normals.argtypes = [ctypes.c_uint64, i64, p]
        L.oracle_max_threads.restype = i32
        for f in ("oracle_quantize_f32", "oracle_quantize_bf16", "oracle_dequantize_bf16",
                  "oracle_qmatmul"):
            getattr(L, f).restype = i32
        _lib = L
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ----------------------------------------------------------------------------- bf16 helpers

def f32_to_bf16_bits(f: np.ndarray) -> np.ndarray:
    """Round-half-to-even narrowing, NaN -> canonical 0x7fff (same rule as the C oracle)."""
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FFF
    return r


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------------------- C oracle

def quantize(w: np.ndarray, bits: int):
    """``QuantizedArray::quantize`` (mlx.rs:1861): [n,k] -> (wq u32, scales bf16 bits, biases bf16 bits)."""
    n, k = w.shape
    wq = np.zeros((n, k * bits // 32), np.uint32)
    s = np.zeros((n, k // GROUP), np.uint16)
    b = np.zeros((n, k // GROUP), np.uint16)
    if w.dtype == np.float32:
        w = np.ascontiguousarray(w)
        rc = lib().oracle_quantize_f32(_ptr(w), n, k, bits, _ptr(wq), _ptr(s), _ptr(b))
    elif w.dtype == np.uint16:  # bf16 bit patterns
        w = np.ascontiguousarray(w)
        rc = lib().oracle_quantize_bf16(_ptr(w), n, k, bits, _ptr(wq), _ptr(s), _ptr(b))
    else:
        raise TypeError(f"oracle.quantize: unsupported dtype {w.dtype}")
    if rc != 0:
        raise ValueError(f"oracle.quantize: invalid shape {w.shape} / bits {bits}")
    return wq, s, b


def dequantize(wq, s, b, n: int, k: int, bits: int) -> np.ndarray:
    """``QuantizedArray::dequantize`` (mlx.rs:1918): bf16 bit patterns [n,k]."""
    out = np.zeros((n, k), np.uint16)
    rc = lib().oracle_dequantize_bf16(_ptr(np.ascontiguousarray(wq)), _ptr(np.ascontiguousarray(s)),
                                      _ptr(np.ascontiguousarray(b)), n, k, bits, _ptr(out))
    if rc != 0:
        raise ValueError("oracle.dequantize: invalid arguments")
    return out


def qmatmul(x_bf16: np.ndarray, wq, s, b, n: int, bits: int, bias_bf16=None, threads: int = 0):
    """``QuantizedArray::matmul`` (mlx.rs:1952): f32 [m,n] = x . dequant(w)^T (+bias), f64 accumulation."""
    m, k = x_bf16.shape
    y = np.zeros((m, n), np.float32)
    x_bf16 = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    bias_bf16 = None if bias_bf16 is None else np.ascontiguousarray(bias_bf16, dtype=np.uint16)
    rc = lib().oracle_qmatmul(_ptr(x_bf16), m, k, _ptr(np.ascontiguousarray(wq)),
                              _ptr(np.ascontiguousarray(s)), _ptr(np.ascontiguousarray(b)), n, bits,
                              _ptr(bias_bf16), _ptr(y), threads)
    if rc != 0:
        raise ValueError("oracle.qmatmul: invalid arguments")
    return y


ACT_NONE, ACT_GELU_TANH, ACT_SILU = 0, 1, 2


def epilogue(acc: np.ndarray, bias_bf16=None, act: int = ACT_NONE, gate_bf16=None, resid_bf16=None):
    """The chains the reference's Flux model builds around a linear, in f64:
    ``resid + gate * act(acc + bias)``.

    * bias: quantized::linear's ``y.add(bias)`` (crates/sd-models/src/mlx/quantized.rs:314-317);
    * act: ``gelu_approx`` = 0.5 a (1 + tanh(sqrt(2/pi) (a + 0.044715 a^3)))
      (crates/sd-tensor/src/mlx.rs:1033-1052) after the MLP's first layer (flux.rs:400-407), or
      ``silu`` = a * sigmoid(a) (mlx.rs:697-705) inside the conditioning MLPs (flux.rs:491-495);
    * gate and resid: ``x.add(&linear(a).mul(&m[2]))`` (flux.rs:389-398, 408-414, 470).
    bias and gate are [n] bf16 bit patterns, resid [m, n]; returns f64 [m, n]."""
    a = acc.astype(np.float64)
    if bias_bf16 is not None:
        a = a + bf16_bits_to_f32(np.asarray(bias_bf16)).astype(np.float64)[None, :]
    if act == ACT_GELU_TANH:
        c = np.sqrt(2.0 / np.pi)
        a = 0.5 * a * (1.0 + np.tanh(c * (a + 0.044715 * a ** 3)))
    elif act == ACT_SILU:
        a = a / (1.0 + np.exp(-a))
    elif act != ACT_NONE:
        raise ValueError(f"oracle.epilogue: unknown activation {act}")
    if gate_bf16 is not None:
        a = a * bf16_bits_to_f32(np.asarray(gate_bf16)).astype(np.float64)[None, :]
    if resid_bf16 is not None:
        a = a + bf16_bits_to_f32(np.asarray(resid_bf16)).astype(np.float64)
    return a


# ---------------------------------------------------------------- GGUF block formats
# The reference's host dequantisation of GGUF tensors (crates/sd-tensor/src/mlx_gguf.rs:235-435),
# restated in NumPy float32 so that every product and difference rounds as the Rust code's does.
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_BF16 = 0, 1, 2, 8, 12, 13, 14, 30
GGML_BLOCKS = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_BF16: (1, 2), GGML_Q4_0: (32, 18), GGML_Q8_0: (32, 34),
               GGML_Q4_K: (256, 144), GGML_Q5_K: (256, 176), GGML_Q6_K: (256, 210)}


def _f16(raw2: np.ndarray) -> np.ndarray:
    """Little-end f16 bytes [..., 2] -> float32 (exact; mlx_gguf.rs:298-318)."""
    return np.ascontiguousarray(raw2).view("<f2")[..., 0].astype(np.float32)


def _scale_min_k4(q: np.ndarray):
    """[blocks, 12] packed bytes -> (scales, mins) [blocks, 8] (mlx_gguf.rs:346-360)."""
    q = q.astype(np.int32)
    sc = np.empty((q.shape[0], 8), np.int32)
    mn = np.empty_like(sc)
    sc[:, :4] = q[:, 0:4] & 63
    mn[:, :4] = q[:, 4:8] & 63
    sc[:, 4:] = (q[:, 8:12] & 0x0F) | ((q[:, 0:4] >> 6) << 4)
    mn[:, 4:] = (q[:, 8:12] >> 4) | ((q[:, 4:8] >> 6) << 4)
    return sc, mn


def gguf_dequantize(raw: np.ndarray, ggml_type: int, count: int) -> np.ndarray:
    """``Gguf::dequantize`` (mlx_gguf.rs:235-283): `count` values of a GGUF tensor as float32."""
    per, nbytes = GGML_BLOCKS[ggml_type]
    if count % per != 0:
        raise ValueError(f"oracle.gguf_dequantize: {count} values are not whole blocks of {per}")
    blocks = count // per
    raw = np.ascontiguousarray(raw, dtype=np.uint8)[: blocks * nbytes].reshape(blocks, nbytes)
    f32 = np.float32
    if ggml_type == GGML_F32:
        return raw.reshape(-1).view("<f4").astype(f32)
    if ggml_type == GGML_F16:
        return raw.reshape(-1).view("<f2").astype(f32)
    if ggml_type == GGML_BF16:
        return (raw.reshape(-1).view("<u2").astype(np.uint32) << 16).view(f32)
    if ggml_type == GGML_Q4_0:                       # mlx_gguf.rs:325-335
        d = _f16(raw[:, 0:2])[:, None]
        qs = raw[:, 2:18].astype(np.int32)
        q = np.concatenate([(qs & 0x0F) - 8, (qs >> 4) - 8], axis=1).astype(f32)
        return (d * q).reshape(-1)
    if ggml_type == GGML_Q8_0:                       # mlx_gguf.rs:337-344
        d = _f16(raw[:, 0:2])[:, None]
        return (d * raw[:, 2:34].view(np.int8).astype(f32)).reshape(-1)
    if ggml_type in (GGML_Q4_K, GGML_Q5_K):          # mlx_gguf.rs:362-410
        d = _f16(raw[:, 0:2])[:, None]
        dmin = _f16(raw[:, 2:4])[:, None]
        sc, mn = _scale_min_k4(raw[:, 4:16])
        d1 = (d * sc.astype(f32))                    # [blocks, 8]
        m1 = (dmin * mn.astype(f32))
        qs = raw[:, 16:144] if ggml_type == GGML_Q4_K else raw[:, 48:176]
        qs = qs.astype(np.int32).reshape(blocks, 4, 32)
        q = np.empty((blocks, 8, 32), np.int32)
        q[:, 0::2] = qs & 0x0F
        q[:, 1::2] = qs >> 4
        if ggml_type == GGML_Q5_K:
            qh = raw[:, 16:48].astype(np.int32)      # [blocks, 32]
            for j in range(8):
                q[:, j] |= ((qh >> j) & 1) << 4
        return (d1[:, :, None] * q.astype(f32) - m1[:, :, None]).reshape(-1)
    if ggml_type == GGML_Q6_K:                       # mlx_gguf.rs:412-435
        ql = raw[:, 0:128].astype(np.int32).reshape(blocks, 2, 64)
        qh = raw[:, 128:192].astype(np.int32).reshape(blocks, 2, 32)
        sc = raw[:, 192:208].view(np.int8).astype(f32).reshape(blocks, 2, 8)
        d = _f16(raw[:, 208:210])[:, None, None]
        out = np.empty((blocks, 2, 4, 32), f32)
        parts = [((ql[:, :, :32] & 0x0F) | ((qh & 3) << 4)) - 32,
                 ((ql[:, :, 32:] & 0x0F) | (((qh >> 2) & 3) << 4)) - 32,
                 ((ql[:, :, :32] >> 4) | (((qh >> 4) & 3) << 4)) - 32,
                 ((ql[:, :, 32:] >> 4) | (((qh >> 6) & 3) << 4)) - 32]
        for quad, q in enumerate(parts):
            # sc[is + 2 quad] with is = l / 16: scales 2 quad and 2 quad + 1 for l < 16 / >= 16
            s = np.repeat(sc[:, :, 2 * quad:2 * quad + 2], 16, axis=2)
            out[:, :, quad, :] = (d * s) * q.astype(f32)
        return out.reshape(-1)
    raise ValueError(f"oracle.gguf_dequantize: unknown GGML type {ggml_type}")


def resident_bytes(n: int, k: int, bits: int, group_size: int = GROUP) -> int:
    return int(lib().oracle_resident_bytes(n, k, group_size, bits))


def seeded_normals(seed: int, count: int) -> np.ndarray:
    """``SeededRng::new(seed).normals(count)`` (lib.rs:104-145)."""
    out = np.zeros(count, np.float32)
    lib().oracle_seeded_normals(ctypes.c_uint64(seed), count, _ptr(out))
    return out


def max_threads() -> int:
    return int(lib().oracle_max_threads())


# ----------------------------------------------------------------------------- NumPy restatement

def _group_extrema(v: np.ndarray):
    """min / max over the last axis under the total order (-0 < +0, NaN ignored)."""
    allnan = np.all(np.isnan(v), axis=-1)
    with np.errstate(invalid="ignore"):
        mn = np.fmin.reduce(v, axis=-1)
        mx = np.fmax.reduce(v, axis=-1)
    neg0 = np.any((v == 0) & np.signbit(v), axis=-1)
    pos0 = np.any((v == 0) & ~np.signbit(v), axis=-1)
    mn = np.where(mn == 0, np.where(neg0, np.float32(-0.0), np.float32(0.0)), mn)
    mx = np.where(mx == 0, np.where(pos0, np.float32(0.0), np.float32(-0.0)), mx)
    mn = np.where(allnan, np.float32(np.inf), mn).astype(np.float32)
    mx = np.where(allnan, np.float32(-np.inf), mx).astype(np.float32)
    return mn, mx


def np_quantize(w: np.ndarray, bits: int):
    """NumPy restatement of the quantiser (same rule, independent code)."""
    w = np.asarray(w, np.float32)
    n, k = w.shape
    assert bits in (4, 8) and k % GROUP == 0
    g = w.reshape(n, k // GROUP, GROUP)
    mn, mx = _group_extrema(g)
    qmax = np.float32((1 << bits) - 1)
    with np.errstate(invalid="ignore", over="ignore"):
        scale = ((mx - mn) / qmax).astype(np.float32)
    sb = f32_to_bf16_bits(scale)
    bb = f32_to_bf16_bits(mn)
    s = bf16_bits_to_f32(sb)[..., None]
    b = bf16_bits_to_f32(bb)[..., None]
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        t = ((g - b) / s).astype(np.float32)
        r = np.rint(t)
    q = np.where(r > 0, np.where(r > qmax, qmax, r), 0)
    q = np.where(np.isnan(r), 0, q)
    q = np.where(s == 0, 0, q).astype(np.uint32)
    per = 32 // bits
    q = q.reshape(n, k // per, per)
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    wq = np.bitwise_or.reduce(q << shifts, axis=-1).astype(np.uint32)
    return wq, sb, bb


def np_dequantize(wq, sb, bb, n: int, k: int, bits: int) -> np.ndarray:
    per = 32 // bits
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    q = ((np.asarray(wq, np.uint32)[..., None] >> shifts) & ((1 << bits) - 1)).reshape(n, k)
    s = np.repeat(bf16_bits_to_f32(sb), GROUP, axis=1)
    b = np.repeat(bf16_bits_to_f32(bb), GROUP, axis=1)
    # s*q is exact in binary32 (<= 16 significant bits), so this is fmaf(s, q, b).
    with np.errstate(invalid="ignore", over="ignore"):
        v = (s * q.astype(np.float32)).astype(np.float32) + b
    return f32_to_bf16_bits(v.astype(np.float32))


# ----------------------------------------------------------------------------- reference generators

def reference_weight(out: int, inp: int) -> np.ndarray:
    """crates/sd-models/tests/mlx_quantized.rs:27-32: ((i % 97) - 48) / 96 as f32."""
    i = np.arange(out * inp, dtype=np.int64)
    return ((np.float32(1.0) * (i % 97).astype(np.float32) - np.float32(48.0)) / np.float32(96.0)
            ).astype(np.float32).reshape(out, inp)


def reference_activation(rows: int, inp: int) -> np.ndarray:
    """crates/sd-models/tests/mlx_quantized.rs:34-39: ((i % 31) - 15) / 15 as f32."""
    i = np.arange(rows * inp, dtype=np.int64)
    return (((i % 31).astype(np.float32) - np.float32(15.0)) / np.float32(15.0)
            ).astype(np.float32).reshape(rows, inp)


def cosine(a, b) -> float:
    """f64-accumulated cosine, as mlx_quantized.rs:41-49 insists."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.dot(a, b) / (np.sqrt(np.dot(a, a)) * np.sqrt(np.dot(b, b))))


def synthetic_linear(seed: int, m: int, k: int, n: int, sigma_w: float, sigma_x: float = 1.0):
    """The documented synthetic draw: X first, then W, each SeededRng normals * sigma;
    X narrowed to bf16 (RNE), W kept f32.  Returns (x_bf16_bits [m,k], w_f32 [n,k])."""
    vals = seeded_normals(seed, m * k + n * k)
    x = (vals[: m * k] * np.float32(sigma_x)).astype(np.float32).reshape(m, k)
    w = (vals[m * k:] * np.float32(sigma_w)).astype(np.float32).reshape(n, k)
    return f32_to_bf16_bits(x), w
