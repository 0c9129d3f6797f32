"""The quantised linear's other consumers: text-encoder layers and Flux's conditioning MLPs.

Shapes only -- these models run the same op (``QuantizedArray::matmul`` through
``quantized::linear``) at their own widths, and this module lists those widths so that the
op can be checked and measured there:

* T5-XXL (``google/t5-v1_1-xxl``, crates/sd-models/src/mlx/t5.rs:41-47): d_model 4096,
  64 heads of 64, d_ff 10240; q/k/v/o without biases and a gated-GELU feed-forward
  ``wo(gelu_new(wi_0(x)) * wi_1(x))`` (t5.rs:185-213).
* The decoder-only encoders of crates/sd-models/src/mlx/llm.rs:70-132 -- Qwen3-4B (Z-Image),
  Qwen2.5-VL-7B's text half (Qwen-Image), Mistral Small 3.2 (FLUX.2): grouped-query
  attention q/k/v/o and a SwiGLU MLP ``down(silu(gate(x)) * up(x))`` (llm.rs:226-291).
* Flux's conditioning MLPs and final modulation at M = 1 (crates/sd-models/src/mlx/flux.rs:
  491-502 mlp_embedder, 525-555 its three uses, 580-585 the output head's modulation):
  time_in / guidance_in (256 -> 3072 -> 3072), vector_in (768 -> 3072 -> 3072),
  final_layer.adaLN_modulation (3072 -> 6144).

Text encoders run on 256 or 512 prompt tokens, so M is 256 or 512.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Tuple

Linear = Tuple[str, int, int, int]      # (weight name, out N, in K, rows M)


@dataclass(frozen=True)
class Encoder:
    name: str
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    layers: int
    ff: str                  # "geglu" (T5) or "swiglu" (the LLMs)
    qkv_bias: bool = False


T5_XXL = Encoder("t5-v1_1-xxl", 4096, 64, 64, 64, 10240, 24, "geglu")
QWEN3_4B = Encoder("qwen3-4b", 2560, 32, 8, 128, 9728, 36, "swiglu")
QWEN2_5_VL_7B = Encoder("qwen2.5-vl-7b", 3584, 28, 4, 128, 18944, 28, "swiglu", qkv_bias=True)
MISTRAL_SMALL_3_2 = Encoder("mistral-small-3.2", 5120, 32, 8, 128, 32768, 40, "swiglu")
ENCODERS = (T5_XXL, QWEN3_4B, QWEN2_5_VL_7B, MISTRAL_SMALL_3_2)


def layer_linears(e: Encoder, tokens: int) -> List[Linear]:
    """The linears of one encoder layer, in execution order."""
    q, kv = e.heads * e.head_dim, e.kv_heads * e.head_dim
    if e.ff == "geglu":
        p = "encoder.block.0.layer"
        attn = [(f"{p}.0.SelfAttention.{n}.weight", q, e.hidden, tokens) for n in ("q", "k", "v")]
        attn.append((f"{p}.0.SelfAttention.o.weight", e.hidden, q, tokens))
        ff = [(f"{p}.1.DenseReluDense.wi_0.weight", e.intermediate, e.hidden, tokens),
              (f"{p}.1.DenseReluDense.wi_1.weight", e.intermediate, e.hidden, tokens),
              (f"{p}.1.DenseReluDense.wo.weight", e.hidden, e.intermediate, tokens)]
        return attn + ff
    p = "model.layers.0"
    attn = [(f"{p}.self_attn.q_proj.weight", q, e.hidden, tokens),
            (f"{p}.self_attn.k_proj.weight", kv, e.hidden, tokens),
            (f"{p}.self_attn.v_proj.weight", kv, e.hidden, tokens),
            (f"{p}.self_attn.o_proj.weight", e.hidden, q, tokens)]
    ff = [(f"{p}.mlp.gate_proj.weight", e.intermediate, e.hidden, tokens),
          (f"{p}.mlp.up_proj.weight", e.intermediate, e.hidden, tokens),
          (f"{p}.mlp.down_proj.weight", e.hidden, e.intermediate, tokens)]
    return attn + ff


def flux_conditioning(hidden: int = 3072, vec_dim: int = 768, time_dim: int = 256) -> List[Linear]:
    """Flux's M = 1 linears outside the blocks: the three conditioning MLPs and the final
    layer's modulation."""
    t: List[Linear] = []
    for mlp, k in (("time_in", time_dim), ("guidance_in", time_dim), ("vector_in", vec_dim)):
        t += [(f"{mlp}.in_layer.weight", hidden, k, 1), (f"{mlp}.out_layer.weight", hidden, hidden, 1)]
    t.append(("final_layer.adaLN_modulation.1.weight", 2 * hidden, hidden, 1))
    return t


def flops(table: List[Linear]) -> float:
    return float(sum(2 * m * n * k for _, n, k, m in table))
