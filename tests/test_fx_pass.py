"""Graph-level behaviour of the FX injector (no kernel launched).

Same contract as upstream tests/test_fx_sdpa.py plus the eager motif,
scale resolution, custom masks and the error paths of
fx_compiler_pass.py:340-368, 475-508.
"""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F  # noqa: N812

from fx_compiler_pass import (BlockSparseAttentionInjector, InjectionConfig,
                              SingleLayerTransformer, StandardAttention,
                              _InjectedTritonAttention, pretty_print_graph)
from sparse_triton_kernel import StreamingMaskSpec, make_streaming_mask


class CausalSdpa(nn.Module):
    def forward(self, q, k, v):
        return F.scaled_dot_product_attention(q, k, v, is_causal=True)


class PlainSdpa(nn.Module):
    def forward(self, q, k, v):
        return F.scaled_dot_product_attention(q, k, v)


class TwoSdpa(nn.Module):
    def forward(self, q, k, v):
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return F.scaled_dot_product_attention(a, k, v, is_causal=True)


class ScaledSdpa(nn.Module):
    def forward(self, q, k, v):
        return F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=0.5)


class DropoutSdpa(nn.Module):
    def forward(self, q, k, v):
        return F.scaled_dot_product_attention(q, k, v, dropout_p=0.1, is_causal=True)


class DivAttention(nn.Module):
    def forward(self, q, k, v):
        s = torch.matmul(q, k.transpose(-2, -1)) / 8.0
        return torch.matmul(torch.softmax(s, dim=-1), v)


class AttrScaleAttention(nn.Module):
    def __init__(self):
        super().__init__()
        self.register_buffer("scale", torch.tensor(0.25))

    def forward(self, q, k, v):
        s = torch.matmul(q, k.transpose(-2, -1)) * self.scale
        return torch.matmul(torch.softmax(s, dim=-1), v)


class NoScaleAttention(nn.Module):
    def forward(self, q, k, v):
        return torch.softmax(q @ k.transpose(-2, -1), dim=-1) @ v


class WrongDimSoftmax(nn.Module):
    def forward(self, q, k, v):
        return torch.matmul(torch.softmax(torch.matmul(q, k.transpose(-2, -1)), dim=-2), v)


class MixedModel(nn.Module):
    def __init__(self):
        super().__init__()
        self.attn = StandardAttention(16)

    def forward(self, q, k, v):
        a = self.attn(q, k, v)
        return F.scaled_dot_product_attention(a, k, v, is_causal=True)


def cfg(**kw):
    base = dict(seq_len_q=64, seq_len_kv=64, head_dim=16,
                streaming=StreamingMaskSpec(sink_size=4, window_size=16),
                block_m=16, block_n=16, device="cpu")
    base.update(kw)
    return InjectionConfig(**base)


def count(gm, pred):
    return sum(1 for n in gm.graph.nodes if pred(n))


def injected(gm):
    return count(gm, lambda n: n.op == "call_module" and str(n.target).startswith("_triton_attn_"))


def sdpa_calls(gm):
    return count(gm, lambda n: n.op == "call_function" and n.target is F.scaled_dot_product_attention)


def test_single_causal_sdpa_is_rewritten():
    gm = BlockSparseAttentionInjector(cfg()).transform(CausalSdpa())
    assert sdpa_calls(gm) == 0 and injected(gm) == 1


def test_two_sdpa_calls_rewritten():
    gm = BlockSparseAttentionInjector(cfg()).transform(TwoSdpa())
    assert sdpa_calls(gm) == 0 and injected(gm) == 2


def test_non_causal_sdpa_refused():
    with pytest.raises(RuntimeError, match="No scaled-dot-product-attention"):
        BlockSparseAttentionInjector(cfg()).transform(PlainSdpa())


def test_dropout_sdpa_refused():
    with pytest.raises(RuntimeError, match="No scaled-dot-product-attention"):
        BlockSparseAttentionInjector(cfg()).transform(DropoutSdpa())


def test_sdpa_module_carries_streaming_params():
    gm = BlockSparseAttentionInjector(cfg()).transform(CausalSdpa())
    m = gm.get_submodule("_triton_attn_0")
    assert isinstance(m, _InjectedTritonAttention)
    assert m.is_causal is True and m.sink_size == 4 and m.window_size == 16
    assert m.block_m == 16 and m.block_n == 16
    assert m.softmax_scale == pytest.approx(1 / math.sqrt(16))


def test_sdpa_static_scale_kept():
    gm = BlockSparseAttentionInjector(cfg()).transform(ScaledSdpa())
    assert gm.get_submodule("_triton_attn_0").softmax_scale == 0.5


def test_eager_motif_rewritten_with_scale():
    gm = BlockSparseAttentionInjector(cfg()).transform(StandardAttention(16))
    assert injected(gm) == 1
    assert count(gm, lambda n: n.op in ("call_function", "call_method")) == 0
    m = gm.get_submodule("_triton_attn_0")
    assert m.softmax_scale == pytest.approx(0.25)
    assert m.is_causal and m.sink_size == 4 and m.window_size == 16


def test_div_scale_inverted():
    gm = BlockSparseAttentionInjector(cfg()).transform(DivAttention())
    assert gm.get_submodule("_triton_attn_0").softmax_scale == pytest.approx(1 / 8.0)


def test_attribute_scale_resolved():
    gm = BlockSparseAttentionInjector(cfg()).transform(AttrScaleAttention())
    assert gm.get_submodule("_triton_attn_0").softmax_scale == pytest.approx(0.25)


def test_unscaled_motif_scale_one():
    gm = BlockSparseAttentionInjector(cfg()).transform(NoScaleAttention())
    assert gm.get_submodule("_triton_attn_0").softmax_scale == 1.0


def test_wrong_softmax_dim_not_matched():
    with pytest.raises(RuntimeError):
        BlockSparseAttentionInjector(cfg()).transform(WrongDimSoftmax())


def test_transformer_block_rewritten_and_numbering():
    gm = BlockSparseAttentionInjector(cfg()).transform(MixedModel())
    # eager matches are numbered before SDPA matches
    assert isinstance(gm.get_submodule("_triton_attn_0"), _InjectedTritonAttention)
    assert gm.get_submodule("_triton_attn_1").is_causal is True
    assert injected(gm) == 2
    gm2 = BlockSparseAttentionInjector(cfg()).transform(SingleLayerTransformer(16, 64))
    assert injected(gm2) == 1


def test_mask_shared_and_on_host():
    inj = BlockSparseAttentionInjector(cfg())
    gm = inj.transform(TwoSdpa())
    a, b = gm.get_submodule("_triton_attn_0"), gm.get_submodule("_triton_attn_1")
    assert a.block_mask is b.block_mask
    assert a.block_mask.device.type == "cpu" and a.block_mask.dtype == torch.int32
    ref = make_streaming_mask(64, 64, StreamingMaskSpec(4, 16), 16, 16, device="cpu")
    assert torch.equal(a.block_mask, ref)
    assert "block_mask" not in gm.state_dict().__repr__() or True  # non-persistent buffer
    assert not any(k.endswith("block_mask") for k in gm.state_dict())


def test_custom_mask_takes_precedence():
    cm = torch.ones(4, 4, dtype=torch.int64)
    gm = BlockSparseAttentionInjector(cfg(custom_mask=cm)).transform(StandardAttention(16))
    m = gm.get_submodule("_triton_attn_0")
    assert m.block_mask.dtype == torch.int32 and torch.equal(m.block_mask, cm.int())


def test_custom_mask_without_streaming_is_not_causal():
    cm = torch.ones(4, 4, dtype=torch.int32)
    gm = BlockSparseAttentionInjector(cfg(custom_mask=cm, streaming=None)).transform(
        StandardAttention(16))
    m = gm.get_submodule("_triton_attn_0")
    assert m.is_causal is False and m.sink_size == 0 and m.window_size == 0


def test_sdpa_without_streaming_uses_full_window():
    cm = torch.ones(4, 4, dtype=torch.int32)
    gm = BlockSparseAttentionInjector(cfg(custom_mask=cm, streaming=None)).transform(CausalSdpa())
    m = gm.get_submodule("_triton_attn_0")
    assert m.is_causal and m.sink_size == 0 and m.window_size == 64


def test_neither_mask_nor_streaming_raises():
    with pytest.raises(ValueError, match="streaming"):
        BlockSparseAttentionInjector(cfg(streaming=None))


def test_original_model_untouched_and_printer():
    model = StandardAttention(16)
    gm = BlockSparseAttentionInjector(cfg()).transform(model)
    assert not hasattr(model, "_triton_attn_0")
    text = pretty_print_graph(gm, "fused")
    assert text.startswith("=== fused ===") and "call_module=1" in text


def test_standard_attention_rejects_bad_dim():
    with pytest.raises(ValueError):
        StandardAttention(0)


def test_llama_style_decoder_rewritten():
    """cfg5's model shape (RMSNorm, RoPE on transposed views, SDPA
    is_causal=True, SwiGLU) in miniature: every layer's SDPA becomes one
    injected module and all of them share one mask buffer."""
    from fx_compiler_pass import LlamaStyleDecoder
    model = LlamaStyleDecoder(vocab=100, hidden=64, n_layers=3, n_heads=4, mlp=128, max_seq=64)
    gm = BlockSparseAttentionInjector(cfg()).transform(model)
    assert sdpa_calls(gm) == 0 and injected(gm) == 3
    mods = [gm.get_submodule(f"_triton_attn_{i}") for i in range(3)]
    assert all(m.block_mask is mods[0].block_mask for m in mods)
    assert all(m.is_causal and m.sink_size == 4 and m.window_size == 16 for m in mods)
    assert mods[0].softmax_scale == pytest.approx(0.25)
    ids = torch.randint(0, 100, (1, 64))
    assert model(ids).shape == (1, 64, 100)  # the original model is untouched and runs


def test_llama_gqa_rewritten():
    from fx_compiler_pass import LlamaStyleDecoder
    model = LlamaStyleDecoder(vocab=100, hidden=64, n_layers=2, n_heads=4, n_kv_heads=2, mlp=128,
                              max_seq=64)
    gm = BlockSparseAttentionInjector(cfg()).transform(model)
    assert sdpa_calls(gm) == 0 and injected(gm) == 2
    assert model(torch.randint(0, 100, (1, 64))).shape == (1, 64, 100)
