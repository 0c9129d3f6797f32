"""sdq -- B200-native affine group-wise quantised linear (host-side mirror).

This package mirrors the reference's `sd-tensor` seam for quantised weights,
``QuantizedArray::{quantize, dequantize, matmul, resident_bytes}``
(andreinknv/stable-diffusion.rs, crates/sd-tensor/src/mlx.rs:1846-1986), over
the C ABI of ``libsdq.so`` (include/sdq.h).  Tensors are torch CUDA tensors used
purely as device memory; every computation is a libsdq kernel.  There is no
CPU fallback: on a machine without an sm_100 device the calls raise
:class:`SdqError`.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from ._abi import (SDQ_BF16, SDQ_ERR_CUDA, SDQ_ERR_INVALID, SDQ_ERR_NCCL, SDQ_ERR_TIMEOUT,
                   SDQ_ERR_UNSUPPORTED, SDQ_F16, SDQ_F32, SDQ_OK, SdqError, check, last_error, lib)

__all__ = [
    "SdqError", "QuantizedArray", "quantize", "dequantize", "quantized_matmul", "quantized_matmul_epilogue",
    "gguf_quantize", "gguf_dequantize", "seeded_normals", "resident_bytes", "ACT_NONE", "ACT_GELU_TANH", "ACT_SILU",
    "device_status", "Comm", "quantized_matmul_sharded", "shard_rows", "unshard", "GROUP_SIZE", "MODE",
    "SDQ_OK", "SDQ_ERR_INVALID", "SDQ_ERR_UNSUPPORTED", "SDQ_ERR_CUDA", "SDQ_ERR_TIMEOUT",
    "SDQ_ERR_NCCL",
]

#: MLX's default group size (crates/sd-models/src/mlx/quantized.rs:45-46).
GROUP_SIZE = 64
#: The quantisation mode the reference always asks for (mlx.rs:1830-1832).
MODE = "affine"

#: Activations of the fused output stage (include/sdq.h SDQ_ACT_*).
ACT_NONE, ACT_GELU_TANH, ACT_SILU = 0, 1, 2
_ACTS = {None: ACT_NONE, "none": ACT_NONE, "gelu_approx": ACT_GELU_TANH, "gelu_tanh": ACT_GELU_TANH,
         "silu": ACT_SILU, ACT_NONE: ACT_NONE, ACT_GELU_TANH: ACT_GELU_TANH, ACT_SILU: ACT_SILU}

_DT = {torch.float32: SDQ_F32, torch.bfloat16: SDQ_BF16, torch.float16: SDQ_F16}


def _dt(t: torch.Tensor) -> int:
    if t.dtype not in _DT:
        raise SdqError(SDQ_ERR_UNSUPPORTED, f"dtype {t.dtype} has no libsdq code")
    return _DT[t.dtype]


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream) -> ctypes.c_void_p:
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise SdqError(SDQ_ERR_INVALID, "libsdq takes device tensors (no CPU fallback)")
        if t is not None and not t.is_contiguous():
            raise SdqError(SDQ_ERR_INVALID, "libsdq takes contiguous row-major tensors")


def quantize(w: torch.Tensor, group_size: int = GROUP_SIZE, bits: int = 4, stream=None,
             sb_dtype=torch.bfloat16):
    """``mlx_quantize`` replacement: w [n, k] f32/bf16 -> (wq u32 [n, k*bits/32] as int32,
    scales [n, k/64], biases [n, k/64]).

    ``sb_dtype`` is bf16 (half the bytes) or f32 (the dtype MLX gives an f32 weight's scales);
    the values are the same bf16-rounded ones either way, widened exactly when f32."""
    _need_cuda(w)
    if sb_dtype not in (torch.bfloat16, torch.float32):
        raise SdqError(SDQ_ERR_UNSUPPORTED, f"scales and biases must be bf16 or f32, not {sb_dtype}")
    if w.dim() != 2:
        raise SdqError(SDQ_ERR_INVALID, f"quantize wants a 2-D weight, got shape {tuple(w.shape)}")
    n, k = w.shape
    if bits not in (4, 8) or k % GROUP_SIZE != 0:
        # Let the library produce the canonical message and code.
        dummy = torch.empty(1, device=w.device, dtype=torch.int32)
        check(lib().sdq_quantize(_ptr(w), _dt(w), n, k, group_size, bits, MODE.encode(), _ptr(dummy),
                                 _ptr(dummy), _ptr(dummy), SDQ_BF16, _stream(stream)))
    wq = torch.empty((n, k * bits // 32), device=w.device, dtype=torch.int32)
    s = torch.empty((n, k // GROUP_SIZE), device=w.device, dtype=sb_dtype)
    b = torch.empty_like(s)
    check(lib().sdq_quantize(_ptr(w), _dt(w), n, k, group_size, bits, MODE.encode(), _ptr(wq), _ptr(s),
                             _ptr(b), _DT[sb_dtype], _stream(stream)))
    return wq, s, b


def dequantize(wq, scales, biases, group_size: int = GROUP_SIZE, bits: int = 4,
               out_dtype=None, stream=None) -> torch.Tensor:
    """``mlx_dequantize`` replacement: reconstruct [n, k] (one rounding of s*q + b).  The
    output dtype defaults to the scales' dtype, as MLX's does (mlx.rs:1935-1938)."""
    _need_cuda(wq, scales, biases)
    if out_dtype is None:
        out_dtype = scales.dtype
    n = wq.shape[0]
    k = wq.shape[1] * 32 // bits
    out = torch.empty((n, k), device=wq.device, dtype=out_dtype)
    check(lib().sdq_dequantize(_ptr(wq), _ptr(scales), _ptr(biases), _dt(scales), n, k, group_size, bits,
                               MODE.encode(), _ptr(out), _dt(out), _stream(stream)))
    return out


def quantized_matmul(x: torch.Tensor, wq, scales, biases, group_size: int = GROUP_SIZE, bits: int = 4,
                     bias: torch.Tensor | None = None, out: torch.Tensor | None = None,
                     stream=None) -> torch.Tensor:
    """``mlx_quantized_matmul`` replacement (transpose=true): x [..., k] -> [..., n].

    A 3-D ``x`` ([b, s, k]) is flattened to M = b*s rows, as MLX does.  ``x``, the scales and
    the result may each be bf16 or f32; the result defaults to ``x``'s dtype.  f32 inputs are
    rounded to bf16 for the tensor cores; an f32 result is the f32 accumulator, unrounded."""
    _need_cuda(x, wq, scales, biases, bias, out)
    lead = x.shape[:-1]
    k = x.shape[-1]
    m = 1
    for d in lead:
        m *= d
    n = wq.shape[0]
    if out is None:
        out = torch.empty((*lead, n), device=x.device,
                          dtype=torch.float32 if x.dtype == torch.float32 else torch.bfloat16)
    check(lib().sdq_quantized_matmul(_ptr(x), _dt(x), m, k, _ptr(wq), _ptr(scales), _ptr(biases),
                                     _dt(scales), n, 1, group_size, bits, MODE.encode(), _ptr(bias),
                                     _ptr(out), _dt(out), _stream(stream)))
    return out


def quantized_matmul_host(x_host: torch.Tensor, wq, scales, biases, group_size: int = GROUP_SIZE,
                          bits: int = 4, bias: torch.Tensor | None = None, out: torch.Tensor | None = None,
                          x_dev: torch.Tensor | None = None, y_dev: torch.Tensor | None = None,
                          chunk_rows: int = 0, stream=None) -> torch.Tensor:
    """:func:`quantized_matmul` on HOST activations into a HOST result (``sdq_quantized_matmul_host``):
    the rows go up, through the product and back down in overlapped chunks.  ``x_host`` and
    ``out`` are CPU tensors (pinned for the copies to overlap); ``x_dev`` / ``y_dev`` are the
    device workspaces (allocated here when not given).  Asynchronous on ``stream``."""
    _need_cuda(wq, scales, biases, bias, x_dev, y_dev)
    if x_host.is_cuda or not x_host.is_contiguous():
        raise SdqError(SDQ_ERR_INVALID, "x_host must be a contiguous CPU tensor")
    lead = x_host.shape[:-1]
    k = x_host.shape[-1]
    m = 1
    for d in lead:
        m *= d
    n = wq.shape[0]
    ydt = torch.float32 if x_host.dtype == torch.float32 else torch.bfloat16
    if out is None:
        out = torch.empty((*lead, n), dtype=ydt, pin_memory=True)
    if out.is_cuda or not out.is_contiguous():
        raise SdqError(SDQ_ERR_INVALID, "out must be a contiguous CPU tensor")
    dev = wq.device
    if x_dev is None:
        x_dev = torch.empty((m, k), device=dev, dtype=x_host.dtype)
    if y_dev is None:
        y_dev = torch.empty((m, n), device=dev, dtype=out.dtype)
    if x_dev.numel() < m * k or y_dev.numel() < m * n or x_dev.dtype != x_host.dtype or y_dev.dtype != out.dtype:
        raise SdqError(SDQ_ERR_INVALID, "x_dev / y_dev must hold m*k / m*n values of x_host's / out's dtype")
    check(lib().sdq_quantized_matmul_host(_ptr(x_host), _dt(x_host), m, k, _ptr(wq), _ptr(scales), _ptr(biases),
                                          _dt(scales), n, group_size, bits, _ptr(bias), _ptr(out), _dt(out),
                                          _ptr(x_dev), _ptr(y_dev), chunk_rows, _stream(stream)))
    return out


def quantized_matmul_epilogue(x: torch.Tensor, wq, scales, biases, group_size: int = GROUP_SIZE,
                              bits: int = 4, bias: torch.Tensor | None = None, act=None,
                              gate: torch.Tensor | None = None, residual: torch.Tensor | None = None,
                              out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """``residual + gate * act(x . dequant(w)^T + bias)`` in one kernel, rounded to bf16 once.

    Replaces the reference's ``x.add(&linear(a).mul(gate))`` and ``linear(a).gelu_approx()`` /
    ``.silu()`` chains (crates/sd-models/src/mlx/flux.rs:389-414, 470, 491-495).  ``act`` is
    None, ``"gelu_approx"`` or ``"silu"`` (or an ``ACT_*`` value); ``gate`` and ``bias`` hold
    ``n`` values (any leading 1-sized dims, as a modulation vector has), ``residual`` has the
    output's shape.  ``out`` may be ``residual`` itself (an in-place residual update)."""
    if act not in _ACTS:
        raise SdqError(SDQ_ERR_INVALID, f"unknown activation {act!r}")
    _need_cuda(x, wq, scales, biases, bias, gate, residual, out)
    lead = x.shape[:-1]
    k = x.shape[-1]
    m = 1
    for d in lead:
        m *= d
    n = wq.shape[0]
    for name, t in (("bias", bias), ("gate", gate)):
        if t is not None and t.numel() != n:
            raise SdqError(SDQ_ERR_INVALID, f"{name} holds {t.numel()} values, the layer has {n} outputs")
    if residual is not None and residual.numel() != m * n:
        raise SdqError(SDQ_ERR_INVALID, f"residual of shape {tuple(residual.shape)} is not [{m}, {n}]")
    if out is None:
        out = torch.empty((*lead, n), device=x.device, dtype=torch.bfloat16)
    check(lib().sdq_quantized_matmul_epilogue(
        _ptr(x), _dt(x), m, k, _ptr(wq), _ptr(scales), _ptr(biases), _dt(scales), n, group_size, bits,
        _ptr(bias), _ACTS[act], _ptr(gate), _ptr(residual), _ptr(out), _dt(out), _stream(stream)))
    return out


def gguf_quantize(raw: torch.Tensor, ggml_type: int, n: int, k: int, bits: int = 4,
                  group_size: int = GROUP_SIZE, stream=None):
    """A GGUF tensor's raw block bytes (uint8 device tensor) -> (wq, scales, biases) of its
    row-major [n, k], bit-identical to quantising its f32 dequantisation (``sdq_gguf_quantize``)."""
    _need_cuda(raw)
    wq = torch.empty((n, k * bits // 32), device=raw.device, dtype=torch.int32)
    s = torch.empty((n, k // GROUP_SIZE), device=raw.device, dtype=torch.bfloat16)
    b = torch.empty_like(s)
    need = int(lib().sdq_gguf_bytes(ggml_type, n * k))
    if need and raw.numel() * raw.element_size() < need:
        raise SdqError(SDQ_ERR_INVALID, f"gguf_quantize: {raw.numel()} bytes, the tensor needs {need}")
    check(lib().sdq_gguf_quantize(_ptr(raw), ggml_type, n, k, group_size, bits, _ptr(wq), _ptr(s), _ptr(b),
                                  SDQ_BF16, _stream(stream)))
    return wq, s, b


def gguf_dequantize(raw: torch.Tensor, ggml_type: int, shape, out_dtype=torch.float32,
                    stream=None) -> torch.Tensor:
    """A GGUF tensor's raw block bytes (uint8 device tensor) -> its values, f32 exactly as the
    reference's host dequantisation gives them, or bf16 (``sdq_gguf_dequantize``)."""
    _need_cuda(raw)
    count = 1
    for d in shape:
        count *= d
    need = int(lib().sdq_gguf_bytes(ggml_type, count))
    if need and raw.numel() * raw.element_size() < need:
        raise SdqError(SDQ_ERR_INVALID, f"gguf_dequantize: {raw.numel()} bytes, the tensor needs {need}")
    out = torch.empty(tuple(shape), device=raw.device, dtype=out_dtype)
    check(lib().sdq_gguf_dequantize(_ptr(raw), ggml_type, count, _ptr(out), _dt(out), _stream(stream)))
    return out


def seeded_normals(seed: int, count: int, device=None, stream=None) -> torch.Tensor:
    """``SeededRng::new(seed).normals(count)`` (crates/sd-tensor/src/lib.rs:104-145) on the
    device, as f32: the reference's documented draw for synthetic inputs."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    out = torch.empty(count, device=dev, dtype=torch.float32)
    check(lib().sdq_seeded_normals(ctypes.c_uint64(seed), count, _ptr(out), _stream(stream)))
    return out


def resident_bytes(n: int, k: int, bits: int, group_size: int = GROUP_SIZE, sb_bytes: int = 4) -> int:
    """Packed words plus scales and biases; ``sb_bytes=4`` counts them as the reference does
    (mlx.rs:1981-1985), ``sb_bytes=2`` is what this library actually stores."""
    return int(lib().sdq_resident_bytes(n, k, group_size, bits, sb_bytes))


def device_status(stream=None) -> None:
    """Raise :class:`SdqError` (SDQ_ERR_TIMEOUT) if a kernel's bounded wait gave up."""
    check(lib().sdq_device_status(_stream(stream)))


def debug_wait_hook(wait_limit_ns: int = 0, withhold_first_copy: bool = False, stream=None) -> None:
    """Testing hook (``sdq_debug_wait_hook``): shorten the kernels' bounded waits to
    ``wait_limit_ns`` (0 restores 2 s) and, with ``withhold_first_copy``, make every CTA's
    weight producer skip its first copy so that the abort path runs."""
    check(lib().sdq_debug_wait_hook(ctypes.c_uint64(wait_limit_ns), int(bool(withhold_first_copy)),
                                    _stream(stream)))


@dataclass
class QuantizedArray:
    """A weight held quantised at rest (mlx.rs:1846-1854): packed ``weight`` (u32 words,
    ``32 / bits`` values each), ``scales``, ``biases``, ``group_size``, ``bits``.

    ``bits`` and ``group_size`` must match what the weight was quantised with; nothing in the
    tensors records them (mlx.rs:1842-1845)."""
    weight: torch.Tensor
    scales: torch.Tensor
    biases: torch.Tensor
    group_size: int
    bits: int

    @classmethod
    def quantize(cls, w: torch.Tensor, group_size: int = GROUP_SIZE, bits: int = 4, stream=None,
                 sb_dtype=torch.bfloat16):
        """``[out, in]`` in, packed ``[out, in * bits / 32]`` out (mlx.rs:1861)."""
        wq, s, b = quantize(w, group_size, bits, stream, sb_dtype)
        return cls(wq, s, b, group_size, bits)

    def dequantize(self, out_dtype=None, stream=None) -> torch.Tensor:
        """Reconstruct the dense array -- for tests, not the hot path (mlx.rs:1913-1918)."""
        return dequantize(self.weight, self.scales, self.biases, self.group_size, self.bits,
                          out_dtype, stream)

    def matmul(self, x: torch.Tensor, bias: torch.Tensor | None = None, stream=None,
               out: torch.Tensor | None = None) -> torch.Tensor:
        """``x @ weight.T``, dequantising inside the kernel (mlx.rs:1947-1975); ``out``, if
        given, receives the result."""
        return quantized_matmul(x, self.weight, self.scales, self.biases, self.group_size, self.bits,
                                bias=bias, out=out, stream=stream)

    def matmul_fused(self, x: torch.Tensor, bias=None, act=None, gate=None, residual=None,
                     out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """``residual + gate * act(x @ weight.T + bias)`` in one kernel (see
        :func:`quantized_matmul_epilogue`)."""
        return quantized_matmul_epilogue(x, self.weight, self.scales, self.biases, self.group_size,
                                         self.bits, bias=bias, act=act, gate=gate, residual=residual,
                                         out=out, stream=stream)

    def resident_bytes(self) -> int:
        """Bytes this weight occupies, counted as the reference does (4 bytes per scale)."""
        packed = self.weight.numel() * 4
        sb = (self.scales.numel() + self.biases.numel()) * 4
        return packed + sb

    @property
    def shape(self):
        return (self.weight.shape[0], self.weight.shape[1] * 32 // self.bits)


class Comm:
    """A libsdq-owned NCCL communicator for the column-sharded linear."""

    def __init__(self, unique_id: bytes, world: int, rank: int):
        if len(unique_id) != 128:
            raise SdqError(SDQ_ERR_INVALID, "NCCL unique id must be 128 bytes")
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(unique_id)
        h = ctypes.c_void_p()
        check(lib().sdq_comm_init(buf, world, rank, ctypes.byref(h)))
        self.handle = h
        self.world = world
        self.rank = rank

    @staticmethod
    def unique_id() -> bytes:
        buf = (ctypes.c_uint8 * 128)()
        check(lib().sdq_comm_unique_id(buf))
        return bytes(buf)

    def output(self, m: int, n: int) -> torch.Tensor:
        """The communicator's output buffer as an [m, n] bf16 tensor (``sdq_comm_output``):
        passed as ``out`` of :func:`quantized_matmul_sharded`, the result is assembled there
        with no final copy.  Collective (same m, n on every rank).  The tensor does not own the
        memory: it is valid until a larger output is asked for or the communicator is destroyed,
        and every sharded call overwrites it."""
        p = ctypes.c_void_p()
        check(lib().sdq_comm_output(self.handle, m, n, ctypes.byref(p)))
        return torch.as_tensor(_DeviceMemory(p.value, (m, n)),
                               device=torch.device("cuda", torch.cuda.current_device())).view(torch.bfloat16)

    def destroy(self) -> None:
        if self.handle:
            check(lib().sdq_comm_destroy(self.handle))
            self.handle = None


class _DeviceMemory:
    """Library-owned device memory seen through the CUDA array interface (int16 elements)."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<i2", "data": (ptr, False),
                                         "version": 3, "strides": None}


def shard_rows(n_total: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [start, stop) of an [n_total, k] weight held by `rank` in the column-sharded
    linear; n_total must divide evenly (every rank runs the same kernel shape)."""
    if n_total % world != 0:
        raise SdqError(SDQ_ERR_INVALID, f"{n_total} output features do not split over {world} ranks")
    nl = n_total // world
    return rank * nl, (rank + 1) * nl


def unshard(y_shards):
    """The permute the library applies after the all-gather: [world, m, n_local] -> [m, world*n_local]
    (host-side statement of the same index map, for arrays or tensors)."""
    w, m, nl = y_shards.shape
    if hasattr(y_shards, "permute"):
        return y_shards.permute(1, 0, 2).reshape(m, w * nl)
    return y_shards.transpose(1, 0, 2).reshape(m, w * nl)


def quantized_matmul_sharded(x, wq, scales, biases, comm: Comm, group_size: int = GROUP_SIZE,
                             bits: int = 4, bias=None, y_shards=None, out=None, permute: bool = True,
                             stream=None):
    """Column-sharded quantised linear: local rows of W -> all-gathered Y [m, world * n_local].

    Returns ``(out, y_shards)``; ``out`` is None when ``permute`` is False (the caller then
    reads the blocked [world, m, n_local] layout from ``y_shards``)."""
    _need_cuda(x, wq, scales, biases, bias)
    m, k = x.reshape(-1, x.shape[-1]).shape
    nl = wq.shape[0]
    if y_shards is None:
        y_shards = torch.empty((comm.world, m, nl), device=x.device, dtype=torch.bfloat16)
    if permute and out is None:
        out = torch.empty((m, comm.world * nl), device=x.device, dtype=torch.bfloat16)
    check(lib().sdq_quantized_matmul_sharded(
        _ptr(x), _dt(x), m, k, _ptr(wq), _ptr(scales), _ptr(biases), _dt(scales), nl, group_size, bits,
        _ptr(bias), _ptr(y_shards), _ptr(out) if permute else None, SDQ_BF16, comm.handle,
        _stream(stream)))
    return (out if permute else None), y_shards
