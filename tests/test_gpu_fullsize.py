"""Parity at the benchmark configurations' full sizes.

The dense oracle does not fit at these sizes, so each test checks a
size-independent property: rows of the forward output against the exact
visible-key computation (a row's output depends only on its visible keys),
and one full (batch, head) slice of forward + gradients against the dense
oracle run on the GPU (the mask is shared by all heads, so one slice
exercises every tile kind).  Tolerance: max-abs <= 2e-2 and rel-L2 <= 5e-3
(bf16/fp16, fixed bounds, against float64 or float32).
"""

from __future__ import annotations

import math

import pytest
import torch

import sbfa_native as native
import sparse_triton_kernel as stk
from fx_compiler_pass import BlockSparseAttentionInjector, InjectionConfig, StandardAttention
from oracle import streaming_oracle as orc
from tests.parity import check_half

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _close(got, ref, label="", dtype=torch.bfloat16):
    check_half(got, ref, dtype, label)


def _gen(shape, dtype, seed, mul=1.0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randn(shape, generator=g, device=DEV, dtype=dtype) * mul


def test_cfg2_fwd_bwd_full_size():
    """B=4, H=32, N=16384, D=128, bf16, S=4, W=2048, BM=BN=128."""
    B, H, N, D, S, W, bm = 4, 32, 16384, 128, 4, 2048, 128
    g = torch.Generator(device=DEV).manual_seed(0)
    q, k, v = (torch.randn(B, H, N, D, generator=g, device=DEV, dtype=torch.bfloat16)
               for _ in range(3))
    do = _gen((B, H, N, D), torch.bfloat16, 1)
    mask = stk.make_streaming_mask(N, N, stk.StreamingMaskSpec(S, W), bm, bm, DEV)
    qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = stk.block_sparse_attention(qq, kk, vv, mask, block_m=bm, block_n=bm, is_causal=True,
                                   sink_size=S, window_size=W)
    o.backward(do)
    assert native.device_status() == 0
    scale = 1 / math.sqrt(D)
    # sampled rows of every head: first rows, window edge, diagonal, last rows
    rows = [0, 1, 127, 128, 2047, 2048, 2049, 9000, N - 129, N - 1]
    for b in range(B):
        for h in range(0, H, 7):
            ro, _ = orc.streaming_rows_forward(q[b, h], k[b, h], v[b, h], rows, S, W, scale)
            _close(o[b, h, rows].detach(), ro, f"O rows b{b} h{h}")
    # one full slice, forward and all three gradients, dense oracle in fp32 on GPU
    b, h = 3, 31
    ro, rdq, rdk, rdv = orc.attention_forward_backward(
        q[b:b + 1, h:h + 1].float(), k[b:b + 1, h:h + 1].float(), v[b:b + 1, h:h + 1].float(),
        do[b:b + 1, h:h + 1].float(), mask.cpu(), block_m=bm, block_n=bm, is_causal=True,
        sink_size=S, window_size=W)
    _close(o[b, h].detach(), ro[0, 0], "O slice")
    _close(qq.grad[b, h], rdq[0, 0], "dQ slice")
    _close(kk.grad[b, h], rdk[0, 0], "dK slice")
    _close(vv.grad[b, h], rdv[0, 0], "dV slice")


def test_cfg3_fwd_full_size():
    """B=1, H=32, N=131072, D=128, fp16 x0.5, S=4, W=4096, BM=BN=128."""
    B, H, N, D, S, W, bm = 1, 32, 131072, 128, 4, 4096, 128
    g = torch.Generator(device=DEV).manual_seed(0)
    q, k, v = (torch.randn(B, H, N, D, generator=g, device=DEV, dtype=torch.float16) * 0.5
               for _ in range(3))
    mask = stk.make_streaming_mask(N, N, stk.StreamingMaskSpec(S, W), bm, bm, DEV)
    with torch.no_grad():
        o = stk.block_sparse_attention(q, k, v, mask, block_m=bm, block_n=bm, is_causal=True,
                                       sink_size=S, window_size=W)
    assert native.device_status() == 0
    scale = 1 / math.sqrt(D)
    rows = [0, 5, 4095, 4096, 4097, 65536, 100000, N - 128, N - 1]
    for h in range(0, H, 3):
        ro, _ = orc.streaming_rows_forward(q[0, h], k[0, h], v[0, h], rows, S, W, scale)
        _close(o[0, h, rows], ro, f"O rows h{h}", torch.float16)


def test_cfg4_decode_full_size():
    """Batch 64, H=32, D=128, one query at position 100000, fp16 cache of
    100001 tokens (105 GB of K/V), S=4, W=2048."""
    B, H, N, D, S, W = 64, 32, 100001, 128, 4, 2048
    k = _gen((B, H, N, D), torch.float16, 11)
    v = _gen((B, H, N, D), torch.float16, 12)
    q = _gen((B, H, 1, D), torch.float16, 10)
    mask = stk.make_streaming_mask(1, N, stk.StreamingMaskSpec(S, W), 1, 64, DEV)
    with torch.no_grad():
        o = stk.block_sparse_attention(q, k, v, mask, block_m=1, block_n=64, is_causal=True,
                                       sink_size=S, window_size=W)
    torch.cuda.synchronize()
    scale = 1 / math.sqrt(D)
    for b, h in [(0, 0), (0, 31), (17, 5), (63, 31), (40, 16)]:
        ro, _ = orc.streaming_rows_forward(q[b, h], k[b, h], v[b, h], [0], S, W, scale)
        _close(o[b, h], ro, f"decode b{b} h{h}", torch.float16)
    del k, v
    torch.cuda.empty_cache()


def test_cfg1_fx_end_to_end():
    """StandardAttention traced and rewritten by the FX pass, B=1, H=4,
    N=1024, D=64, fp32, S=4, W=256, BM=BN=64: output and dQ/dK/dV against
    eager masked attention (upstream verify tiers: 1e-4 fwd, 1e-3 grads)."""
    cfg = InjectionConfig(seq_len_q=1024, seq_len_kv=1024, head_dim=64,
                          streaming=stk.StreamingMaskSpec(4, 256), block_m=64, block_n=64)
    fused = BlockSparseAttentionInjector(cfg).transform(StandardAttention(64)).to(DEV)
    g = torch.Generator(device=DEV).manual_seed(0)
    q, k, v = (torch.randn(1, 4, 1024, 64, generator=g, device=DEV, requires_grad=True)
               for _ in range(3))
    out = fused(q, k, v)
    gout = _gen(out.shape, torch.float32, 1)
    out.backward(gout)
    ro, rdq, rdk, rdv = orc.attention_forward_backward(
        q.detach().double().cpu(), k.detach().double().cpu(), v.detach().double().cpu(),
        gout.double().cpu(), fused.get_submodule("_triton_attn_0").block_mask.cpu(),
        block_m=64, block_n=64, is_causal=True, sink_size=4, window_size=256)
    assert torch.allclose(out.detach().double().cpu(), ro, atol=1e-4, rtol=1e-4)
    for got, ref in ((q.grad, rdq), (k.grad, rdk), (v.grad, rdv)):
        assert torch.allclose(got.double().cpu(), ref, atol=1e-3, rtol=1e-3)
