"""Quantised-at-rest weights: the per-tensor policy and the dispatching linear.

Mirror of the reference's `sd_models::mlx::quantized`
(crates/sd-models/src/mlx/quantized.rs): the same names, the same rules and
the same errors, with `QuantizedArray` backed by libsdq instead of MLX.  Dense
(non-quantisable) weights keep the reference's dense linear, ``x @ w.T + b``
(crates/sd-models/src/mlx/mod.rs:182-189), on the device.
"""
from __future__ import annotations

from typing import Callable, Dict, Mapping, Optional, Protocol

import torch
import torch.nn.functional as F

from . import ACT_GELU_TANH, ACT_NONE, ACT_SILU, QuantizedArray, SdqError
from ._abi import SDQ_ERR_INVALID

#: MLX's default group size; must divide the weight's input width (quantized.rs:45-46).
GROUP_SIZE = 64
#: Bits per weight by default (quantized.rs:47-49).
DEFAULT_BITS = 4

Weights = Dict[str, torch.Tensor]


class QuantizedWeights:
    """Large weights quantised, the rest dense; both consulted by name (quantized.rs:51-86)."""

    def __init__(self, quantized: Optional[Dict[str, QuantizedArray]] = None,
                 dense: Optional[Weights] = None):
        self.quantized: Dict[str, QuantizedArray] = quantized or {}
        self.dense: Weights = dense or {}

    def resident_bytes(self) -> int:
        """Packed weights plus scales and biases, plus dense tensors at 4 bytes each."""
        q = sum(a.resident_bytes() for a in self.quantized.values())
        d = sum(t.numel() * 4 for t in self.dense.values())
        return q + d

    def __len__(self) -> int:
        return len(self.quantized) + len(self.dense)

    def is_empty(self) -> bool:
        return len(self) == 0

    def contains_key(self, name: str) -> bool:
        return name in self.quantized or name in self.dense

    # WeightSource (quantized.rs:359-380)
    def linear(self, x: torch.Tensor, name: str, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        return linear(x, name, bias, self)

    def linear_fused(self, x: torch.Tensor, name: str, bias: Optional[torch.Tensor] = None, act=None,
                     gate: Optional[torch.Tensor] = None,
                     residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        return linear_fused(x, name, bias, self, act, gate, residual)

    def dense_tensor(self, name: str) -> torch.Tensor:
        if name in self.dense:
            return self.dense[name]
        if name in self.quantized:
            raise SdqError(SDQ_ERR_INVALID, f"mlx: {name} is quantised; reach it through `linear` "
                                            "rather than dequantising it")
        raise SdqError(SDQ_ERR_INVALID, f"mlx: missing tensor {name}")

    def optional(self, name: str) -> Optional[torch.Tensor]:
        return self.dense.get(name)


def sensitive(name: str) -> bool:
    """Layers that get 8 bits whatever the default (quantized.rs:110-117)."""
    return ("_mod.lin" in name or "modulation" in name or "_embedder" in name
            or name.startswith("img_in") or name.startswith("txt_in") or name.startswith("final_layer"))


def indexed(name: str) -> bool:
    """Tensors read by index, never multiplied, so never quantised (quantized.rs:131-152)."""
    return (name == "shared.weight" or "relative_attention_bias" in name or "_embedding.weight" in name
            or name.endswith("pos_embed") or "prd_embedding" in name or "positional_embedding" in name
            or name == "x_embedder.proj.weight" or name == "model.embed_tokens.weight"
            or name == "lm_head.weight")


def mixed(bits: int) -> Callable[[str], int]:
    """Default policy: indexed dense (0), sensitive 8, the rest ``bits`` (quantized.rs:156-166)."""
    def f(name: str) -> int:
        if indexed(name):
            return 0
        if sensitive(name):
            return 8
        return bits
    return f


def quantizable(shape) -> bool:
    """2-D with an input width that divides by the group size (quantized.rs:172-174)."""
    return len(shape) == 2 and shape[1] % GROUP_SIZE == 0


def from_dense(w: Mapping[str, torch.Tensor], bits: int) -> QuantizedWeights:
    """Quantise an already-loaded dense map with the default policy (quantized.rs:265-267)."""
    return from_dense_with(w, mixed(bits))


def from_dense_with(w: Mapping[str, torch.Tensor], bits_for: Callable[[str], int],
                    stream=None) -> QuantizedWeights:
    """``from_dense`` with an explicit per-tensor bit width; 0 keeps a tensor dense
    (quantized.rs:273-291).  Each weight is quantised on the device and the dense
    source may be dropped by the caller right after."""
    quantized: Dict[str, QuantizedArray] = {}
    dense: Weights = {}
    for name, array in w.items():
        bits = bits_for(name)
        if bits >= 2 and quantizable(tuple(array.shape)):
            quantized[name] = QuantizedArray.quantize(array.contiguous(), GROUP_SIZE, bits, stream)
        else:
            dense[name] = array.contiguous()
    return QuantizedWeights(quantized, dense)


def from_gguf(path: str, bits: int, device=None, stream=None) -> QuantizedWeights:
    """Load a GGUF checkpoint, quantising the large weights as they are read
    (quantized.rs:180-211).  One tensor at a time: its raw block bytes are copied to the
    device and either quantised there straight from the block format (``sdq.gguf_quantize``)
    or dequantised to a dense f32 tensor; nothing else of the file is held meanwhile."""
    return _load_gguf(path, bits, None, device, stream)


def from_gguf_renamed(path: str, bits: int, rename: Callable[[str], Optional[str]], device=None,
                      stream=None) -> QuantizedWeights:
    """``from_gguf`` with file names translated by ``rename`` (None drops a tensor),
    quantized.rs:221-255."""
    return _load_gguf(path, bits, rename, device, stream)


def _load_gguf(path, bits, rename, device, stream) -> QuantizedWeights:
    from . import gguf as G
    from . import gguf_dequantize, gguf_quantize

    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    g = G.Gguf(path)
    quantized: Dict[str, QuantizedArray] = {}
    dense: Weights = {}
    policy = mixed(bits)
    for info in g.tensors:
        name = info.name if rename is None else rename(info.name)
        if name is None:
            continue
        raw = torch.from_numpy(g.raw(info)).to(dev)         # the peak: one tensor's blocks
        want = policy(name)
        if want >= 2 and quantizable(info.shape):
            n, k = info.shape
            wq, s, b = gguf_quantize(raw, info.kind, n, k, want, GROUP_SIZE, stream)
            quantized[name] = QuantizedArray(wq, s, b, GROUP_SIZE, want)
        else:
            dense[name] = gguf_dequantize(raw, info.kind, info.shape, torch.float32, stream)
        del raw
    if not quantized and not dense:
        raise SdqError(SDQ_ERR_INVALID, f"gguf: {path} carries no tensors"
                       + ("" if rename is None else " this model recognises"))
    return QuantizedWeights(quantized, dense)


def dense_linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The reference's dense ``x @ w.T + b`` (crates/sd-models/src/mlx/mod.rs:182-189)."""
    y = torch.matmul(x, w.t().to(x.dtype))
    return y if b is None else y + b


def linear(x: torch.Tensor, name: str, bias: Optional[torch.Tensor], w: QuantizedWeights) -> torch.Tensor:
    """``x @ w[name].T + bias`` by whichever kernel suits how ``name`` is held
    (quantized.rs:298-318).  The quantised branch fuses the bias into the kernel's
    epilogue instead of a separate add."""
    q = w.quantized.get(name)
    if q is not None:
        return q.matmul(x, bias=bias)
    d = w.dense.get(name)
    if d is None:
        raise SdqError(SDQ_ERR_INVALID, f"mlx: {name} is in neither map")
    return dense_linear(x, d, bias)


def apply_epilogue(y: torch.Tensor, act=None, gate: Optional[torch.Tensor] = None,
                   residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The elementwise chain after a linear, one op at a time as the reference runs it:
    ``gelu_approx`` / ``silu`` (flux.rs:400-407, 491-495), then ``.mul(gate)`` and
    ``x.add(..)`` (flux.rs:389-398, 408-414, 470)."""
    if act in ("gelu_approx", "gelu_tanh", ACT_GELU_TANH):
        y = F.gelu(y, approximate="tanh")
    elif act in ("silu", ACT_SILU):
        y = F.silu(y)
    elif act not in (None, "none", ACT_NONE):
        raise SdqError(SDQ_ERR_INVALID, f"unknown activation {act!r}")
    if gate is not None:
        y = y * gate
    if residual is not None:
        y = residual + y
    return y


def linear_fused(x: torch.Tensor, name: str, bias: Optional[torch.Tensor], w: QuantizedWeights, act=None,
                 gate: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``residual + gate * act(linear(x))``: one libsdq kernel when ``name`` is quantised, the
    op-by-op chain otherwise."""
    q = w.quantized.get(name)
    if q is not None:
        return q.matmul_fused(x, bias=bias, act=act, gate=gate, residual=residual)
    return apply_epilogue(linear(x, name, bias, w), act, gate, residual)


class OpByOp:
    """A weight source whose ``linear_fused`` runs the linear and then the elementwise chain
    op by op, as the reference does -- for measuring what the fused output stage saves."""

    def __init__(self, inner):
        self.inner = inner

    def linear(self, x, name, bias=None):
        return self.inner.linear(x, name, bias)

    def linear_fused(self, x, name, bias=None, act=None, gate=None, residual=None):
        return apply_epilogue(self.inner.linear(x, name, bias), act, gate, residual)

    def dense_tensor(self, name):
        return self.inner.dense_tensor(name)

    def optional(self, name):
        return self.inner.optional(name)


class WeightSource(Protocol):
    """Where a model's weights come from (quantized.rs:325-339)."""

    def linear(self, x: torch.Tensor, name: str, bias: Optional[torch.Tensor] = None) -> torch.Tensor: ...

    def linear_fused(self, x: torch.Tensor, name: str, bias: Optional[torch.Tensor] = None, act=None,
                     gate: Optional[torch.Tensor] = None,
                     residual: Optional[torch.Tensor] = None) -> torch.Tensor: ...

    def dense_tensor(self, name: str) -> torch.Tensor: ...

    def optional(self, name: str) -> Optional[torch.Tensor]: ...


class DenseWeights(dict):
    """``impl WeightSource for Weights`` (quantized.rs:341-357): every tensor dense."""

    def linear(self, x, name, bias=None):
        if name not in self:
            raise SdqError(SDQ_ERR_INVALID, f"mlx: missing tensor {name}")
        return dense_linear(x, self[name], bias)

    def linear_fused(self, x, name, bias=None, act=None, gate=None, residual=None):
        return apply_epilogue(self.linear(x, name, bias), act, gate, residual)

    def dense_tensor(self, name):
        if name not in self:
            raise SdqError(SDQ_ERR_INVALID, f"mlx: missing tensor {name}")
        return self[name]

    def optional(self, name):
        return self.get(name)
