"""Ring-buffer KV cache on the GPU: the appended rows land where the format
says (byte-exact against the oracle's row map), and decoding over the ring
matches the block-sparse decode over the full-length cache (same visible
keys, different summation order: max-abs <= 2e-3 * max(1, |ref|) in fp32
accumulation) and the oracle's streaming rows."""

from __future__ import annotations

import math

import pytest
import torch

import sbfa_native as native
import sparse_triton_kernel as stk
from oracle import streaming_oracle as orc
from streaming_kv_cache import StreamingKVCache

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _full_decode(q, k, v, L, sink, window):
    mask = stk.make_streaming_mask(1, L, stk.StreamingMaskSpec(sink, window), 1, 64, DEV)
    with torch.no_grad():
        return stk.block_sparse_attention(q, k[:, :, :L], v[:, :, :L], mask, block_m=1,
                                          block_n=64, is_causal=True, sink_size=sink,
                                          window_size=window)


@pytest.mark.parametrize("dtype,D,sink,window,chunks", [
    (torch.float16, 128, 4, 256, [1000, 1, 1, 1, 300, 1, 700, 1]),
    (torch.bfloat16, 64, 4, 64, [3, 1, 1, 100, 1, 64, 65, 1]),
    (torch.float16, 64, 0, 32, [50, 1, 1, 33, 1]),
    (torch.float32, 64, 5, 48, [7, 60, 1, 1]),
    (torch.float16, 128, 3, 0, [10, 1, 1]),
])
def test_ring_matches_full_cache_decode(dtype, D, sink, window, chunks):
    B, H = 2, 3
    total = sum(chunks)
    g = torch.Generator(device=DEV).manual_seed(3)
    k = torch.randn(B, H, total, D, generator=g, device=DEV, dtype=dtype)
    v = torch.randn(B, H, total, D, generator=g, device=DEV, dtype=dtype)
    cache = StreamingKVCache(B, H, D, sink, window, dtype=dtype, device=DEV)
    pos = 0
    for n in chunks:
        cache.append(k[:, :, pos:pos + n], v[:, :, pos:pos + n])
        pos += n
        q = torch.randn(B, H, 1, D, generator=g, device=DEV, dtype=dtype)
        o_ring = cache.attend(q)
        o_full = _full_decode(q, k, v, pos, sink, window)
        err = (o_ring.double() - o_full.double()).abs().max().item()
        assert err <= 2e-3 * max(1.0, o_full.double().abs().max().item()), (pos, err)
        rows = orc.ring_cache_positions(sink, window, pos)
        for r, p in enumerate(rows.tolist()):
            if p >= 0:
                assert torch.equal(cache.k[:, :, r], k[:, :, p]), (r, p)
                assert torch.equal(cache.v[:, :, r], v[:, :, p]), (r, p)
    assert native.device_status() == 0
    # the last step against the oracle's visible-key computation (float64)
    ro, _ = orc.streaming_rows_forward(q[1, 2], k[1, 2, :pos], v[1, 2, :pos], [0], sink, window,
                                       1 / math.sqrt(D))
    assert (o_ring[1, 2].double() - ro.double()).abs().max().item() <= 2e-2


def test_ring_cfg4_memory_and_values():
    """Config-4 geometry (S=4, W=2048, position 100000) on a few heads: the
    ring holds 2052 rows per head instead of 100001 and decodes the same."""
    B, H, D, S, W, L = 2, 4, 128, 4, 2048, 100001
    g = torch.Generator(device=DEV).manual_seed(7)
    k = torch.randn(B, H, L, D, generator=g, device=DEV, dtype=torch.float16)
    v = torch.randn(B, H, L, D, generator=g, device=DEV, dtype=torch.float16)
    cache = StreamingKVCache(B, H, D, S, W, dtype=torch.float16, device=DEV)
    cache.append(k, v)
    assert cache.memory_bytes * (L / (S + W)) == pytest.approx(2 * k.numel() * 2, rel=1e-9)
    q = torch.randn(B, H, 1, D, generator=g, device=DEV, dtype=torch.float16)
    o_ring, lse_ring = cache.attend(q, return_lse=True)
    o_full = _full_decode(q, k, v, L, S, W)
    assert (o_ring.double() - o_full.double()).abs().max().item() <= 2e-3
    assert torch.isfinite(lse_ring).all()
