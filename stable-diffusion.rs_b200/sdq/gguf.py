"""GGUF container reader (and a small writer), the host side of the load-time pipeline.

Mirror of the reference's ``sd_tensor::mlx_gguf::Gguf`` (crates/sd-tensor/src/mlx_gguf.rs:
150-233): the same checks (magic, versions 2 and 3, the supported type set), metadata skipped,
shapes reversed to row-major, tensor data starting at the next 32-byte boundary (or at
``general.alignment`` when the file declares one).  The block data of a tensor is handed out
raw; ``sdq.gguf_quantize`` / ``sdq.gguf_dequantize`` decode it on the GPU.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np

from ._abi import SDQ_ERR_INVALID, SDQ_ERR_UNSUPPORTED, SdqError

MAGIC = 0x46554747                                     # "GGUF", little-end
F32, F16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 2, 8, 12, 13, 14, 30
#: (values per block, bytes per block), mlx_gguf.rs:25-40, 80-93.
BLOCKS = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144),
          Q5_K: (256, 176), Q6_K: (256, 210)}
NAMES = {F32: "F32", F16: "F16", BF16: "BF16", Q4_0: "Q4_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K",
         Q6_K: "Q6_K"}
_SCALAR = {0: 1, 1: 1, 7: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 10: 8, 11: 8, 12: 8}   # metadata value sizes


@dataclass
class TensorInfo:
    name: str
    shape: Tuple[int, ...]      # row-major (the file writes fastest-varying first)
    kind: int
    offset: int                 # from the start of the data section

    def elem_count(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n

    def nbytes(self) -> int:
        per, b = BLOCKS[self.kind]
        return self.elem_count() // per * b


class _Reader:
    def __init__(self, f):
        self.f = f

    def take(self, fmt: str):
        size = struct.calcsize(fmt)
        b = self.f.read(size)
        if len(b) != size:
            raise SdqError(SDQ_ERR_INVALID, "gguf: unexpected end of file")
        return struct.unpack(fmt, b)[0]

    def string(self) -> str:
        n = self.take("<Q")
        b = self.f.read(n)
        try:
            return b.decode("utf-8")
        except UnicodeDecodeError as e:
            raise SdqError(SDQ_ERR_INVALID, f"gguf: bad utf8 in a name: {e}") from e

    def value(self, kind: int):
        """Read one metadata value (kept only for general.alignment; the rest is skipped)."""
        if kind in _SCALAR:
            fmt = {1: {0: "<B", 1: "<b", 7: "<?"}, 2: {2: "<H", 3: "<h"}, 4: {4: "<I", 5: "<i", 6: "<f"},
                   8: {10: "<Q", 11: "<q", 12: "<d"}}[_SCALAR[kind]][kind]
            return self.take(fmt)
        if kind == 8:
            return self.string()
        if kind == 9:
            inner, count = self.take("<I"), self.take("<Q")
            for _ in range(count):
                self.value(inner)
            return None
        raise SdqError(SDQ_ERR_INVALID, f"gguf: unknown metadata type {kind}")


class Gguf:
    """The tensor directory of a GGUF file and where its data starts (``Gguf::open``)."""

    def __init__(self, path: str):
        self.path = path
        with open(path, "rb") as f:
            r = _Reader(f)
            if r.take("<I") != MAGIC:
                raise SdqError(SDQ_ERR_INVALID, f"gguf: {path} is not a GGUF file")
            version = r.take("<I")
            if version not in (2, 3):
                raise SdqError(SDQ_ERR_UNSUPPORTED, f"gguf: version {version} is not supported")
            n_tensors, n_kv = r.take("<Q"), r.take("<Q")
            self.alignment = 32
            for _ in range(n_kv):
                key = r.string()
                v = r.value(r.take("<I"))
                if key == "general.alignment" and isinstance(v, int) and v > 0:
                    self.alignment = v
            self.tensors: List[TensorInfo] = []
            for _ in range(n_tensors):
                name = r.string()
                dims = [r.take("<Q") for _ in range(r.take("<I"))]
                kind = r.take("<I")
                if kind not in BLOCKS:
                    raise SdqError(SDQ_ERR_UNSUPPORTED,
                                   f"gguf: type {kind} is not one this project's checkpoints use; the "
                                   "supported set is F32, F16, BF16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K")
                self.tensors.append(TensorInfo(name, tuple(reversed(dims)), kind, r.take("<Q")))
            here = f.tell()
        self.data_start = (here + self.alignment - 1) // self.alignment * self.alignment

    def raw(self, info: TensorInfo) -> np.ndarray:
        """The tensor's block bytes (mlx_gguf.rs:237-252: whole blocks or an error)."""
        per, _ = BLOCKS[info.kind]
        if info.elem_count() % per != 0:
            raise SdqError(SDQ_ERR_INVALID,
                           f"gguf: {info.name} has {info.elem_count()} elements, not a multiple of {per}")
        data = np.fromfile(self.path, dtype=np.uint8, count=info.nbytes(), offset=self.data_start + info.offset)
        if data.size != info.nbytes():
            raise SdqError(SDQ_ERR_INVALID, f"gguf: {info.name}'s data runs past the end of the file")
        return data


def write(path: str, tensors: Iterable[Tuple[str, Sequence[int], int, np.ndarray]],
          metadata: Optional[Dict[str, int]] = None, alignment: int = 32) -> None:
    """Write a GGUF v3 file of (name, row-major shape, type, raw block bytes) tensors, with
    optional u32 metadata.  For tests and tools; the reference only reads GGUF."""
    tensors = list(tensors)
    meta = dict(metadata or {})
    if alignment != 32:
        meta["general.alignment"] = alignment

    def s(x: str) -> bytes:
        b = x.encode("utf-8")
        return struct.pack("<Q", len(b)) + b

    head = struct.pack("<IIQQ", MAGIC, 3, len(tensors), len(meta))
    for k, v in meta.items():
        head += s(k) + struct.pack("<II", 4, v)
    offsets, off = [], 0
    for name, shape, kind, raw in tensors:
        offsets.append(off)
        off += (len(raw) + alignment - 1) // alignment * alignment
    for (name, shape, kind, raw), o in zip(tensors, offsets):
        head += s(name) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in reversed(shape))
        head += struct.pack("<IQ", kind, o)
    pad = (-len(head)) % alignment
    with open(path, "wb") as f:
        f.write(head + b"\0" * pad)
        for (_, _, _, raw), o in zip(tensors, offsets):
            b = np.ascontiguousarray(raw, dtype=np.uint8).tobytes()
            f.write(b + b"\0" * ((-len(b)) % alignment))
