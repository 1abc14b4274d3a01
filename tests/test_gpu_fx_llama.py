"""The FX pass on a Llama-style decoder (the cfg5 model family) in
miniature, bf16 on the GPU: logits and parameter gradients of the rewritten
model against the same model with the StreamingLLM token mask applied through
torch's masked SDPA.  Only attention differs between the two, so the
tolerance is tight: rel-L2 <= 1e-2 for logits, loss and every gradient."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F  # noqa: N812

import sparse_triton_kernel as stk
from fx_compiler_pass import BlockSparseAttentionInjector, InjectionConfig, LlamaStyleDecoder

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("n_kv_heads", [2, 1])
def test_llama_fx_end_to_end_matches_masked_sdpa(monkeypatch, n_kv_heads):
    """n_kv_heads = 1: grouped-query attention (enable_gqa=True) through the
    same pass and kernels."""
    torch.manual_seed(0)
    n, sink, window = 1024, 4, 256
    model = LlamaStyleDecoder(vocab=512, hidden=256, n_layers=2, n_heads=2, mlp=512, max_seq=n,
                              n_kv_heads=n_kv_heads, device=DEV, dtype=torch.bfloat16)
    cfg = InjectionConfig(seq_len_q=n, seq_len_kv=n, head_dim=128,
                          streaming=stk.StreamingMaskSpec(sink, window), block_m=64, block_n=64)
    fused = BlockSparseAttentionInjector(cfg).transform(model).to(DEV)
    g = torch.Generator(device=DEV).manual_seed(1)
    ids = torch.randint(0, 512, (2, n), generator=g, device=DEV)
    tgt = torch.randint(0, 512, (2, n), generator=g, device=DEV)

    def step(m):
        for p in model.parameters():
            p.grad = None
        logits = m(ids)
        loss = F.cross_entropy(logits.float().view(-1, 512), tgt.view(-1))
        loss.backward()
        return logits.detach(), loss.detach(), {k: p.grad.clone() for k, p in
                                                model.named_parameters()}

    lf, lossf, gf = step(fused)
    tok = stk.streaming_token_mask(n, n, sink, window, device=DEV)
    orig = F.scaled_dot_product_attention

    def masked_sdpa(q, k, v, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None, **kw):
        return orig(q, k, v, attn_mask=tok, dropout_p=dropout_p, scale=scale, **kw)

    monkeypatch.setattr(torch.nn.functional, "scaled_dot_product_attention", masked_sdpa)
    lr, lossr, gr = step(model)
    assert torch.isfinite(lf).all()
    assert _rel(lf, lr) <= 1e-2
    assert abs(lossf.item() - lossr.item()) <= 1e-2 * abs(lossr.item())
    for k in gr:
        assert torch.isfinite(gf[k]).all(), k
        assert _rel(gf[k], gr[k]) <= 1e-2, (k, _rel(gf[k], gr[k]))
