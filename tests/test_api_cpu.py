"""Host-side behaviour of the drop-in ``sparse_triton_kernel`` module.

Covers what upstream pins on CPU (tests/test_streaming_definition.py,
tests/test_mask_equivalence.py, tests/test_oracle.py): the mask builders
against the golden fixtures and a by-hand definition of the StreamingLLM
rule, block-mask ⊇ token-mask, and the error behaviour of the autograd
bridge when no CUDA tensors are given.
"""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import sparse_triton_kernel as stk
from oracle import streaming_oracle as orc
from tests.golden.make_golden import BLOCK_CASES, DENSE_CASES, TOKEN_CASES, key_block


def _by_hand(n_q, n_kv, sink, window):
    """Position-by-position StreamingLLM rule; no helper from either module."""
    out = np.zeros((n_q, n_kv), dtype=bool)
    for r in range(n_q):
        qa = n_kv - n_q + r
        for ka in range(n_kv):
            out[r, ka] = ka <= qa and (ka < sink or qa - ka < window)
    return out


@pytest.fixture(scope="module")
def masks(golden_dir):
    return np.load(os.path.join(golden_dir, "block_masks.npz"))


def _unpack(masks, key):
    shape = tuple(masks[key + "_shape"].tolist())
    n = int(np.prod(shape))
    return np.unpackbits(masks[key + "_bits"])[:n].reshape(shape).astype(np.int32)


@pytest.mark.parametrize("case", BLOCK_CASES, ids=key_block)
def test_host_streaming_mask_matches_golden(masks, case):
    n_q, n_kv, s, w, bm, bn = case
    got = stk.make_streaming_mask(n_q, n_kv, stk.StreamingMaskSpec(s, w), bm, bn, device="cpu")
    assert got.dtype == torch.int32 and got.is_contiguous()
    assert np.array_equal(got.numpy(), _unpack(masks, key_block(case)))


@pytest.mark.parametrize("case", DENSE_CASES)
def test_host_dense_mask_matches_golden(masks, case):
    n_q, n_kv, bm, bn, causal = case
    got = stk.make_dense_mask(n_q, n_kv, bm, bn, causal=causal, device="cpu")
    key = "dense_" + "_".join(str(int(x)) for x in case)
    assert np.array_equal(got.numpy(), _unpack(masks, key))


@pytest.mark.parametrize("case", [c for c in TOKEN_CASES if c[0] * c[1] <= 70_000])
def test_token_mask_matches_hand_definition(case):
    got = stk.streaming_token_mask(*case, device="cpu").numpy()
    assert np.array_equal(got, _by_hand(*case))


def test_decode_query_sees_sink_plus_window():
    m = stk.streaming_token_mask(1, 1000, 4, 256)
    assert int(m.sum()) == 4 + 256


def test_sink_never_sees_the_future():
    m = stk.streaming_token_mask(4, 4, 4, 1).numpy()
    assert np.array_equal(m, np.tril(np.ones((4, 4), dtype=bool)))


@pytest.mark.parametrize("case", [c for c in BLOCK_CASES if c[0] * c[1] <= 2_000_000])
def test_block_mask_covers_token_mask(case):
    n_q, n_kv, s, w, bm, bn = case
    bmask = stk.make_streaming_mask(n_q, n_kv, stk.StreamingMaskSpec(s, w), bm, bn, "cpu")
    lifted = orc.lift_block_mask(bmask.numpy(), n_q, n_kv, bm, bn)
    tok = orc.streaming_token_mask(n_q, n_kv, s, w)
    assert not np.any(tok & ~lifted)
    # lifted & token == token: the kernel's effective mask is the paper's
    assert np.array_equal(lifted & tok, tok)


def test_lifted_block_mask_alone_is_looser():
    """Without the in-block token rule the diagonal blocks leak."""
    bmask = stk.make_streaming_mask(32, 32, stk.StreamingMaskSpec(4, 8), 8, 8, "cpu")
    lifted = orc.lift_block_mask(bmask.numpy(), 32, 32, 8, 8)
    assert np.any(lifted & ~orc.streaming_token_mask(32, 32, 4, 8))


def test_spec_rejects_negative():
    with pytest.raises(ValueError, match="non-negative"):
        stk.StreamingMaskSpec(-1, 4)


def test_streaming_mask_rejects_empty():
    with pytest.raises(ValueError, match="positive"):
        stk.make_streaming_mask(0, 10, stk.StreamingMaskSpec(1, 1), 2, 2, device="cpu")


def test_dense_mask_requires_divisible():
    with pytest.raises(ValueError, match="divide"):
        stk.make_dense_mask(10, 10, 3, 2, device="cpu")


def test_eager_function_matches_oracle_fp64():
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 2, 48, 16, generator=g, dtype=torch.float64)
    k = torch.randn(1, 2, 80, 16, generator=g, dtype=torch.float64)
    v = torch.randn(1, 2, 80, 16, generator=g, dtype=torch.float64)
    m = stk.make_streaming_mask(48, 80, stk.StreamingMaskSpec(4, 16), 16, 16, "cpu")
    a = stk.reference_block_sparse_attention(q, k, v, m, block_m=16, block_n=16,
                                             is_causal=True, sink_size=4, window_size=16)
    b = orc.attention_forward(q, k, v, m, block_m=16, block_n=16, is_causal=True,
                              sink_size=4, window_size=16)
    assert torch.allclose(a, b, atol=1e-12, rtol=1e-12)


def test_bridge_rejects_host_tensors():
    q = torch.randn(1, 1, 16, 16)
    m = torch.ones(1, 1, dtype=torch.int32)
    with pytest.raises((ValueError, RuntimeError)):
        stk.block_sparse_attention(q, q, q, m, block_m=16, block_n=16)


def test_bridge_rejects_wrong_rank():
    q = torch.randn(1, 16, 16)
    with pytest.raises((ValueError, RuntimeError)):
        stk.block_sparse_attention(q, q, q, torch.ones(1, 1, dtype=torch.int32))
