"""Host logic of the quantised-weight policy, mirrored from
crates/sd-models/src/mlx/quantized.rs (pure string / shape rules, no device)."""
from __future__ import annotations

import pytest

from sdq import quantized as Q


@pytest.mark.parametrize("name", [
    "double_blocks.0.img_mod.lin.weight", "double_blocks.3.txt_mod.lin.weight",
    "single_blocks.7.modulation.lin.weight", "time_in.in_layer.weight".replace("time_in", "t_embedder"),
    "img_in.weight", "txt_in.weight", "final_layer.linear.weight", "final_layer.adaLN_modulation.1.weight",
])
def test_sensitive_layers(name):
    assert Q.sensitive(name)
    assert Q.mixed(4)(name) == 8


@pytest.mark.parametrize("name", [
    "double_blocks.0.img_attn.qkv.weight", "double_blocks.0.img_attn.proj.weight",
    "double_blocks.0.img_mlp.0.weight", "single_blocks.3.linear1.weight", "single_blocks.3.linear2.weight",
])
def test_ordinary_layers_take_the_default(name):
    assert not Q.sensitive(name) and not Q.indexed(name)
    assert Q.mixed(4)(name) == 4
    assert Q.mixed(8)(name) == 8


@pytest.mark.parametrize("name", [
    "shared.weight", "encoder.block.0.layer.0.SelfAttention.relative_attention_bias.weight",
    "token_embedding.weight".replace("token", "x_token"), "pos_embed", "prd_embedding",
    "positional_embedding", "x_embedder.proj.weight", "model.embed_tokens.weight", "lm_head.weight",
])
def test_indexed_tensors_stay_dense(name):
    assert Q.indexed(name)
    assert Q.mixed(4)(name) == 0


def test_quantizable_rule():
    """2-D and K % 64 == 0 (quantized.rs:172-174); norms, biases and odd widths stay dense."""
    assert Q.quantizable((128, 256))
    assert not Q.quantizable((128,))        # a bias / norm
    assert not Q.quantizable((32, 100))     # 100 does not divide by 64
    assert not Q.quantizable((2, 3, 64))
    assert Q.GROUP_SIZE == 64 and Q.DEFAULT_BITS == 4
