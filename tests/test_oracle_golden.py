"""Pin the CPU oracle to outputs of the upstream reference itself.

The fixtures under ``tests/golden/`` were produced by
``tests/golden/make_golden.py`` running the upstream
``sparse_triton_kernel.py``; these tests check ``oracle/`` reproduces
them bit-exactly (masks) or to 1e-12 in float64 (attention and grads).
"""

from __future__ import annotations

import hashlib
import json
import os

import numpy as np
import pytest
import torch

from oracle import streaming_oracle as orc
from tests.golden.make_golden import (ATTN_CASES, ATTN_TC_CASES, BLOCK_CASES, DENSE_CASES,
                                      TOKEN_CASES, key_block)


@pytest.fixture(scope="module")
def masks(golden_dir):
    return np.load(os.path.join(golden_dir, "block_masks.npz"))


@pytest.fixture(scope="module")
def attn(golden_dir):
    return np.load(os.path.join(golden_dir, "attention_cases.npz"))


def _unpack(masks, key):
    shape = tuple(masks[key + "_shape"].tolist())
    n = int(np.prod(shape))
    return np.unpackbits(masks[key + "_bits"])[:n].reshape(shape).astype(np.int32)


@pytest.mark.parametrize("case", BLOCK_CASES, ids=key_block)
def test_streaming_block_mask_bit_exact(masks, case):
    n_q, n_kv, s, w, bm, bn = case
    got = orc.make_streaming_mask(n_q, n_kv, s, w, bm, bn)
    want = _unpack(masks, key_block(case))
    assert got.dtype == np.int32 and got.shape == want.shape
    assert np.array_equal(got, want)
    assert int(got.sum()) == int(masks[key_block(case) + "_nnz"])


@pytest.mark.parametrize("case", DENSE_CASES)
def test_dense_block_mask_bit_exact(masks, case):
    n_q, n_kv, bm, bn, causal = case
    got = orc.make_dense_mask(n_q, n_kv, bm, bn, causal)
    key = "dense_" + "_".join(str(int(x)) for x in case)
    assert np.array_equal(got, _unpack(masks, key))


@pytest.mark.parametrize("case", TOKEN_CASES)
def test_token_mask_matches_reference(golden_dir, case):
    with open(os.path.join(golden_dir, "token_masks.json")) as fh:
        tok = json.load(fh)
    want = tok["_".join(str(x) for x in case)]
    m = orc.streaming_token_mask(*case)
    assert int(m.sum()) == want["popcount"]
    assert hashlib.sha256(m.sum(axis=1).astype(np.int64).tobytes()).hexdigest() == \
        want["row_counts_sha256"]
    assert hashlib.sha256(np.packbits(m.ravel()).tobytes()).hexdigest() == want["bits_sha256"]


@pytest.mark.parametrize("name", [c[0] for c in ATTN_CASES])
def test_attention_forward_backward_matches_reference(attn, name):
    p = f"{name}__"
    B, H, n_q, n_kv, D, bm, bn, causal, s, w = attn[p + "params"].tolist()
    t = {k: torch.from_numpy(attn[p + k]) for k in ("q", "k", "v", "do", "o", "dq", "dk", "dv")}
    o, dq, dk, dv = orc.attention_forward_backward(
        t["q"], t["k"], t["v"], t["do"], attn[p + "mask"], block_m=bm, block_n=bn,
        is_causal=bool(causal), sink_size=s, window_size=w)
    for nm, got in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv)):
        assert torch.allclose(got, t[nm], atol=1e-12, rtol=1e-12), nm


def tc_case_inputs(g, name: str):
    """Inputs of a tensor-core golden case as tensors of their 16-bit type,
    plus the case parameters and the stored float32 reference outputs."""
    p = f"{name}__"
    params = g[p + "params"].tolist()
    dt = getattr(torch, str(g[p + "dtype"]))
    ins = {k: torch.from_numpy(g[p + k]).view(dt) for k in ("q", "k", "v", "do")}
    outs = {k: torch.from_numpy(g[p + k]) for k in ("o", "dq", "dk", "dv")}
    return params, dt, g[p + "mask"], ins, outs


@pytest.mark.parametrize("name", [c[0] for c in ATTN_TC_CASES])
def test_tensor_core_cases_match_reference(golden_dir, name):
    """The oracle in float64 on the 16-bit inputs reproduces the upstream
    outputs stored for the tensor-core shapes (stored as float32)."""
    g = np.load(os.path.join(golden_dir, "attention_tc_cases.npz"))
    (B, H, n_q, n_kv, D, bm, bn, causal, s, w), dt, mask, ins, outs = tc_case_inputs(g, name)
    assert dt in (torch.float16, torch.bfloat16) and D in (64, 128) and bm == bn == 128
    o, dq, dk, dv = orc.attention_forward_backward(
        *(ins[k].double() for k in ("q", "k", "v", "do")), mask, block_m=bm, block_n=bn,
        is_causal=bool(causal), sink_size=s, window_size=w)
    for nm, got in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv)):
        assert torch.allclose(got.float(), outs[nm], atol=1e-6, rtol=1e-6), nm


def test_empty_rows_are_zero_in_golden(attn):
    """The fully-masked first query block yields exact zeros (upstream
    tests/test_fully_masked_row.py:160-175)."""
    p = "custom_empty_row__"
    assert np.all(attn[p + "o"][:, :, :16] == 0)
    assert np.all(attn[p + "dq"][:, :, :16] == 0)


def test_tile_plan_flags_and_order():
    m = orc.make_streaming_mask(300, 300, 4, 64, 64, 64)
    plan = orc.tile_plan(m, 300, 300, 64, 64, 128, 128)
    # tile grid 3x3; 128-tiles over 64-blocks: kept iff any covered block kept
    assert plan["row_ptr"].tolist()[0] == 0
    assert int(plan["row_ptr"][-1]) == int(plan["nnz"]) == int(plan["col_ptr"][-1])
    cols = (plan["col_idx"].view(np.uint32) & 0x7FFFFFFF).tolist()
    for i in range(3):
        seg = cols[plan["row_ptr"][i]:plan["row_ptr"][i + 1]]
        assert seg == sorted(seg)
