"""A Flux-schnell-shaped transformer whose every linear is libsdq's quantised matmul.

This is the measurement harness for the whole-model configuration: hidden 3072, 24 heads of
128, MLP ratio 4, 19 double-stream and 38 single-stream blocks, 512 text + 4096 image tokens,
bf16 activations, the residual-multiplying linears (attention out-projection, MLP
down-projection, the single blocks' output projection) at 8 bits and every other linear at 4,
group 64.  The weights are random (no checkpoint exists here).

The block structure, tensor names and the order of operations follow the reference's forward
(crates/sd-models/src/mlx/flux.rs): norm_modulate 255-274, modulation 279-299, split_qkv
302-311, qk_norm 323-329, double_block 333-421, single_block 424-474, timestep_embedding
477-489, mlp_embedder 491-508, forward 510-603, the rotary tables embed_nd 126-157 and the
interleaved rotation rotate 165-212.  What sits between the linears -- LayerNorm, the RMS
query/key norm, the rotary embedding, attention, GELU, SiLU, gates and residuals -- is plain
torch on the device: the callers' arithmetic around the quantised linear, not the path
itself.  Every linear goes through a ``WeightSource`` (``sdq.quantized``), so the same forward
runs on a dense source for comparison.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Dict, Iterator, List, Optional, Tuple

import torch
import torch.nn.functional as F

from . import QuantizedArray
from .quantized import GROUP_SIZE, QuantizedWeights, quantizable

EPS = 1e-6
TIME_EMBED_DIM = 256
TIME_FACTOR = 1000.0


@dataclass(frozen=True)
class FluxShape:
    """Sizes of the stack (defaults: the whole-model configuration)."""

    hidden: int = 3072
    heads: int = 24
    mlp_ratio: float = 4.0
    depth: int = 19
    depth_single: int = 38
    txt_tokens: int = 512
    img_tokens: int = 4096
    in_channels: int = 64
    context_dim: int = 4096
    vec_dim: int = 768
    axes_dim: Tuple[int, ...] = (16, 56, 56)
    theta: float = 10_000.0

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def mlp_hidden(self) -> int:
        return int(self.hidden * self.mlp_ratio)


def linear_table(cfg: FluxShape) -> List[Tuple[str, int, int, int]]:
    """Every linear of one forward, in execution order: (weight name, out, in, rows M)."""
    h, mh, nt, ni = cfg.hidden, cfg.mlp_hidden, cfg.txt_tokens, cfg.img_tokens
    t: List[Tuple[str, int, int, int]] = [
        ("img_in.weight", h, cfg.in_channels, ni),
        ("txt_in.weight", h, cfg.context_dim, nt),
        ("time_in.in_layer.weight", h, TIME_EMBED_DIM, 1),
        ("time_in.out_layer.weight", h, h, 1),
        ("vector_in.in_layer.weight", h, cfg.vec_dim, 1),
        ("vector_in.out_layer.weight", h, h, 1),
    ]
    for i in range(cfg.depth):
        p = f"double_blocks.{i}"
        t += [(f"{p}.img_mod.lin.weight", 6 * h, h, 1), (f"{p}.txt_mod.lin.weight", 6 * h, h, 1)]
        for tag, m in (("img", ni), ("txt", nt)):
            t.append((f"{p}.{tag}_attn.qkv.weight", 3 * h, h, m))
        for tag, m in (("img", ni), ("txt", nt)):
            t += [(f"{p}.{tag}_attn.proj.weight", h, h, m), (f"{p}.{tag}_mlp.0.weight", mh, h, m),
                  (f"{p}.{tag}_mlp.2.weight", h, mh, m)]
    for i in range(cfg.depth_single):
        p = f"single_blocks.{i}"
        t += [(f"{p}.modulation.lin.weight", 3 * h, h, 1), (f"{p}.linear1.weight", 3 * h + mh, h, nt + ni),
              (f"{p}.linear2.weight", h, h + mh, nt + ni)]
    t += [("final_layer.adaLN_modulation.1.weight", 2 * h, h, 1),
          ("final_layer.linear.weight", cfg.in_channels, h, ni)]
    return t


def flops(cfg: FluxShape) -> float:
    """2 M N K summed over every linear of one forward."""
    return float(sum(2 * m * n * k for _, n, k, m in linear_table(cfg)))


def output_stage(name: str) -> Tuple[Optional[str], bool]:
    """(activation, gated residual update) fused into the linear's output stage in forward():
    the MLP's first layer and the conditioning MLPs' inner layer apply an activation, and the
    projections that feed the residual stream multiply by a modulation gate and add into it."""
    if name.endswith("_mlp.0.weight"):
        return "gelu_approx", False
    if name.endswith(".in_layer.weight"):
        return "silu", False
    return None, bits_for(name) == 8


def bits_for(name: str) -> int:
    """The whole-model configuration's policy: residual-multiplying projections 8 bits, the rest 4."""
    if name.endswith("_attn.proj.weight") or name.endswith("_mlp.2.weight") or name.endswith(".linear2.weight"):
        return 8
    return 4


def dense_tensor_table(cfg: FluxShape) -> List[Tuple[str, Tuple[int, ...]]]:
    """The small dense tensors: every linear's bias and the query/key RMS-norm scales."""
    t = [(name[: -len("weight")] + "bias", (n,)) for name, n, _, _ in linear_table(cfg)]
    for i in range(cfg.depth):
        for tag in ("img", "txt"):
            for nm in ("query_norm", "key_norm"):
                t.append((f"double_blocks.{i}.{tag}_attn.norm.{nm}.scale", (cfg.head_dim,)))
    for i in range(cfg.depth_single):
        for nm in ("query_norm", "key_norm"):
            t.append((f"single_blocks.{i}.norm.{nm}.scale", (cfg.head_dim,)))
    return t


def random_weights(cfg: FluxShape, seed: int = 0, device="cuda",
                   bits: Callable[[str], int] = bits_for, keep_dense: bool = False):
    """Random-init weights, each linear drawn on the device, quantised and its dense copy dropped
    before the next (the reference's one-tensor-at-a-time load, quantized.rs:273-291).  W ~ N(0,
    1/K) keeps activations O(1) through the stack.  Returns QuantizedWeights, plus (when
    ``keep_dense``) a dict of the dequantised weights and the dense tensors for comparison."""
    g = torch.Generator(device).manual_seed(seed)
    quantized: Dict[str, QuantizedArray] = {}
    dense: Dict[str, torch.Tensor] = {}
    dq: Dict[str, torch.Tensor] = {}
    for name, n, k, _ in linear_table(cfg):
        w = torch.randn(n, k, device=device, generator=g) / math.sqrt(k)
        assert quantizable(tuple(w.shape))
        q = QuantizedArray.quantize(w, GROUP_SIZE, bits(name))
        quantized[name] = q
        if keep_dense:
            dq[name] = q.dequantize()
        del w
    for name, shape in dense_tensor_table(cfg):
        if name.endswith(".scale"):
            dense[name] = (1.0 + 0.1 * torch.randn(shape, device=device, generator=g)).to(torch.bfloat16)
        else:
            dense[name] = (0.02 * torch.randn(shape, device=device, generator=g)).to(torch.bfloat16)
    qw = QuantizedWeights(quantized, dense)
    if keep_dense:
        dq.update(dense)
        return qw, dq
    return qw


# ---------------------------------------------------------------- the callers' arithmetic
def rope_tables(cfg: FluxShape, device="cuda") -> Tuple[torch.Tensor, torch.Tensor]:
    """cos / sin [seq, head_dim / 2] for text ids (0, 0, 0) then image ids (0, row, col) of a
    square latent grid, one frequency band per axis (flux.rs:89-101, 126-157)."""
    side = int(math.isqrt(cfg.img_tokens))
    assert side * side == cfg.img_tokens, "image tokens must form a square grid"
    rows = torch.arange(side, dtype=torch.float64).repeat_interleave(side)
    cols = torch.arange(side, dtype=torch.float64).repeat(side)
    ids = torch.zeros(cfg.txt_tokens + cfg.img_tokens, 3, dtype=torch.float64)
    ids[cfg.txt_tokens:, 1] = rows
    ids[cfg.txt_tokens:, 2] = cols
    angles = []
    for axis, dim in enumerate(cfg.axes_dim):
        i = torch.arange(dim // 2, dtype=torch.float64)
        omega = 1.0 / cfg.theta ** (2.0 * i / dim)
        angles.append(ids[:, axis:axis + 1] * omega)
    ang = torch.cat(angles, dim=1)
    return ang.cos().float().to(device), ang.sin().float().to(device)


def norm_modulate(x, shift, scale):
    y = F.layer_norm(x.float(), (x.shape[-1],), eps=EPS)
    return (y * (1.0 + scale.float()) + shift.float()).to(torch.bfloat16)


def qk_norm(x, weight):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + EPS) * weight.float()).to(torch.bfloat16)


def rotate(x, cos, sin):
    """Interleaved pairs (x[2i], x[2i+1]) rotated by (cos[i], sin[i]); x is [b, heads, n, d]."""
    b, hh, n, d = x.shape
    xf = x.float().reshape(b, hh, n, d // 2, 2)
    even, odd = xf[..., 0], xf[..., 1]
    c, s = cos.view(1, 1, n, d // 2), sin.view(1, 1, n, d // 2)
    out = torch.stack((even * c - odd * s, even * s + odd * c), dim=-1)
    return out.reshape(b, hh, n, d).to(torch.bfloat16)


def split_qkv(qkv, heads, hd):
    b, n, _ = qkv.shape
    t = qkv.reshape(b, n, 3, heads, hd).permute(2, 0, 3, 1, 4)
    return t[0], t[1], t[2]


def merge_heads(x):
    b, hh, n, d = x.shape
    return x.transpose(1, 2).reshape(b, n, hh * d)


def modulation(w, vec, prefix, n):
    out = w.linear(F.silu(vec), f"{prefix}.lin.weight", w.optional(f"{prefix}.lin.bias"))
    return out.reshape(out.shape[0], 1, -1).chunk(n, dim=-1)


def timestep_embedding(t, dim, theta):
    half = dim // 2
    freqs = torch.exp(-math.log(theta) * torch.arange(half, device=t.device, dtype=torch.float32) / half)
    args = (t.float().reshape(-1, 1) * TIME_FACTOR) * freqs.view(1, half)
    return torch.cat((args.cos(), args.sin()), dim=1).to(torch.bfloat16)


def mlp_embedder(w, x, prefix):
    h = w.linear_fused(x, f"{prefix}.in_layer.weight", w.optional(f"{prefix}.in_layer.bias"), act="silu")
    return w.linear(h, f"{prefix}.out_layer.weight", w.optional(f"{prefix}.out_layer.bias"))


def attention(q, k, v):
    return merge_heads(F.scaled_dot_product_attention(q, k, v, scale=1.0 / math.sqrt(q.shape[-1])))


def double_block(w, img, txt, vec, cos, sin, i, cfg: FluxShape):
    p = f"double_blocks.{i}"
    heads, hd = cfg.heads, cfg.head_dim
    im = modulation(w, vec, f"{p}.img_mod", 6)
    tm = modulation(w, vec, f"{p}.txt_mod", 6)

    def stream_qkv(x, m, tag):
        qkv = w.linear(norm_modulate(x, m[0], m[1]), f"{p}.{tag}_attn.qkv.weight",
                       w.optional(f"{p}.{tag}_attn.qkv.bias"))
        q, k, v = split_qkv(qkv, heads, hd)
        return (qk_norm(q, w.dense_tensor(f"{p}.{tag}_attn.norm.query_norm.scale")),
                qk_norm(k, w.dense_tensor(f"{p}.{tag}_attn.norm.key_norm.scale")), v)

    iq, ik, iv = stream_qkv(img, im, "img")
    tq, tk, tv = stream_qkv(txt, tm, "txt")
    q = rotate(torch.cat((tq, iq), dim=2), cos, sin)
    k = rotate(torch.cat((tk, ik), dim=2), cos, sin)
    v = torch.cat((tv, iv), dim=2)
    a = attention(q, k, v)
    nt = txt.shape[1]

    # x + gate * linear(..) and gelu(linear(..)) run inside the linear's output stage.
    def finish(x, att, m, tag):
        x = w.linear_fused(att.contiguous(), f"{p}.{tag}_attn.proj.weight",
                           w.optional(f"{p}.{tag}_attn.proj.bias"), gate=m[2], residual=x)
        ff = w.linear_fused(norm_modulate(x, m[3], m[4]), f"{p}.{tag}_mlp.0.weight",
                            w.optional(f"{p}.{tag}_mlp.0.bias"), act="gelu_approx")
        return w.linear_fused(ff, f"{p}.{tag}_mlp.2.weight", w.optional(f"{p}.{tag}_mlp.2.bias"),
                              gate=m[5], residual=x)

    return finish(img, a[:, nt:], im, "img"), finish(txt, a[:, :nt], tm, "txt")


def single_block(w, x, vec, cos, sin, i, cfg: FluxShape):
    p = f"single_blocks.{i}"
    h, heads, hd = cfg.hidden, cfg.heads, cfg.head_dim
    m = modulation(w, vec, f"{p}.modulation", 3)
    proj = w.linear(norm_modulate(x, m[0], m[1]), f"{p}.linear1.weight", w.optional(f"{p}.linear1.bias"))
    q, k, v = split_qkv(proj[..., : 3 * h].contiguous(), heads, hd)
    q = rotate(qk_norm(q, w.dense_tensor(f"{p}.norm.query_norm.scale")), cos, sin)
    k = rotate(qk_norm(k, w.dense_tensor(f"{p}.norm.key_norm.scale")), cos, sin)
    joined = torch.cat((attention(q, k, v), F.gelu(proj[..., 3 * h:], approximate="tanh")), dim=2)
    return w.linear_fused(joined, f"{p}.linear2.weight", w.optional(f"{p}.linear2.bias"),
                          gate=m[2], residual=x)


def forward(w, img, txt, timestep, pooled, cfg: FluxShape, rope) -> torch.Tensor:
    """One transformer forward: img [1, n_img, in_channels], txt [1, n_txt, context_dim],
    timestep [1], pooled [1, vec_dim] (bf16) -> [1, n_img, in_channels]."""
    cos, sin = rope
    img = w.linear(img, "img_in.weight", w.optional("img_in.bias"))
    txt = w.linear(txt, "txt_in.weight", w.optional("txt_in.bias"))
    vec = mlp_embedder(w, timestep_embedding(timestep, TIME_EMBED_DIM, cfg.theta), "time_in")
    vec = vec + mlp_embedder(w, pooled, "vector_in")
    for i in range(cfg.depth):
        img, txt = double_block(w, img, txt, vec, cos, sin, i, cfg)
    x = torch.cat((txt, img), dim=1)
    for i in range(cfg.depth_single):
        x = single_block(w, x, vec, cos, sin, i, cfg)
    img = x[:, txt.shape[1]:]
    shift, scale = w.linear(F.silu(vec), "final_layer.adaLN_modulation.1.weight",
                            w.optional("final_layer.adaLN_modulation.1.bias")).reshape(1, 1, -1).chunk(2, dim=-1)
    return w.linear(norm_modulate(img, shift, scale), "final_layer.linear.weight",
                    w.optional("final_layer.linear.bias"))


def inputs(cfg: FluxShape, seed: int = 1, device="cuda"):
    """Seeded synthetic inputs of the forward's shapes."""
    g = torch.Generator(device).manual_seed(seed)
    img = torch.randn(1, cfg.img_tokens, cfg.in_channels, device=device, generator=g).to(torch.bfloat16)
    txt = torch.randn(1, cfg.txt_tokens, cfg.context_dim, device=device, generator=g).to(torch.bfloat16)
    pooled = torch.randn(1, cfg.vec_dim, device=device, generator=g).to(torch.bfloat16)
    timestep = torch.full((1,), 0.5, device=device)
    return img, txt, timestep, pooled


class LinearsOnly:
    """The forward's 312 linears alone, in execution order, on preallocated inputs and outputs:
    the quantised-matmul share of a forward, timed without the surrounding arithmetic."""

    def __init__(self, w: QuantizedWeights, cfg: FluxShape, seed: int = 2, device="cuda"):
        g = torch.Generator(device).manual_seed(seed)
        self.w = w
        self.calls = []
        xs: Dict[Tuple[int, int], torch.Tensor] = {}
        for name, n, k, m in linear_table(cfg):
            if (m, k) not in xs:
                xs[(m, k)] = torch.randn(m, k, device=device, generator=g).to(torch.bfloat16)
            y = torch.empty(m, n, device=device, dtype=torch.bfloat16)
            act, gated = output_stage(name)
            gate = resid = None
            if gated:      # the forward's gate [n] and residual stream [m, n]
                gate = torch.randn(n, device=device, generator=g).to(torch.bfloat16)
                resid = torch.randn(m, n, device=device, generator=g).to(torch.bfloat16)
            self.calls.append((w.quantized[name], xs[(m, k)], w.optional(name[: -len("weight")] + "bias"), y,
                               act, gate, resid))

    def __call__(self) -> None:
        for q, x, b, y, act, gate, resid in self.calls:
            if act is None and gate is None:
                q.matmul(x, bias=b, out=y)
            else:
                q.matmul_fused(x, bias=b, act=act, gate=gate, residual=resid, out=y)

    def __iter__(self) -> Iterator:
        return iter(self.calls)
