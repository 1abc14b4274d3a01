"""GPU mask and plan kernels are bit-exact with the upstream mask builders
(golden fixtures) and with the oracle's tile plans."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import sparse_triton_kernel as stk
from oracle import streaming_oracle as orc
from tests.golden.make_golden import BLOCK_CASES, DENSE_CASES, key_block

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def masks(golden_dir):
    return np.load(os.path.join(golden_dir, "block_masks.npz"))


def _unpack(masks, key):
    shape = tuple(masks[key + "_shape"].tolist())
    n = int(np.prod(shape))
    return np.unpackbits(masks[key + "_bits"])[:n].reshape(shape).astype(np.int32)


@pytest.mark.parametrize("case", BLOCK_CASES, ids=key_block)
def test_gpu_streaming_mask_bit_exact(masks, case):
    n_q, n_kv, s, w, bm, bn = case
    got = stk.make_streaming_mask(n_q, n_kv, stk.StreamingMaskSpec(s, w), bm, bn, device="cuda")
    assert got.is_cuda and got.dtype == torch.int32
    assert np.array_equal(got.cpu().numpy(), _unpack(masks, key_block(case)))


@pytest.mark.parametrize("case", DENSE_CASES)
def test_gpu_dense_mask_bit_exact(masks, case):
    n_q, n_kv, bm, bn, causal = case
    got = stk.make_dense_mask(n_q, n_kv, bm, bn, causal=causal, device="cuda")
    key = "dense_" + "_".join(str(int(x)) for x in case)
    assert np.array_equal(got.cpu().numpy(), _unpack(masks, key))


def _check_plan(mask_np, n_q, n_kv, bm, bn, tm, tn):
    m = torch.from_numpy(mask_np).cuda()
    plan = stk.build_plan(m, n_q, n_kv, bm, bn, tm, tn)
    want = orc.tile_plan(mask_np, n_q, n_kv, bm, bn, tm, tn)
    nnz = int(plan["nnz"].item())
    assert nnz == int(want["nnz"])
    assert np.array_equal(plan["row_ptr"].cpu().numpy(), want["row_ptr"])
    assert np.array_equal(plan["col_ptr"].cpu().numpy(), want["col_ptr"])
    assert np.array_equal(plan["col_idx"][:nnz].cpu().numpy(), want["col_idx"])
    assert np.array_equal(plan["row_idx"][:nnz].cpu().numpy(), want["row_idx"])


PLAN_CASES = [
    # (n_q, n_kv, S, W, bm, bn, tile_m, tile_n)
    (1024, 1024, 4, 256, 64, 64, 128, 128),     # cfg1 mask, 128 tiles over 64 blocks
    (1024, 1024, 4, 256, 64, 64, 16, 64),
    (1024, 1024, 4, 256, 64, 64, 64, 16),
    (1000, 1000, 4, 128, 64, 64, 128, 128),     # ragged
    (1, 1000, 4, 256, 1, 64, 1, 64),            # decode
    (1, 100001, 4, 2048, 1, 64, 1, 64),         # cfg4 decode plan
    (7, 300, 0, 5, 3, 17, 16, 64),              # odd user blocks
    (300, 7, 2, 1, 17, 3, 64, 16),
    (129, 257, 1, 64, 128, 128, 128, 128),
    (2048, 2048, 4, 512, 128, 128, 128, 128),
]


@pytest.mark.parametrize("case", PLAN_CASES)
def test_gpu_plan_matches_oracle(case):
    n_q, n_kv, s, w, bm, bn, tm, tn = case
    m = orc.make_streaming_mask(n_q, n_kv, s, w, bm, bn)
    _check_plan(m, n_q, n_kv, bm, bn, tm, tn)


def test_gpu_plan_random_custom_masks():
    rng = np.random.default_rng(0)
    for n_q, n_kv, bm, bn, tm, tn in [(96, 160, 32, 32, 16, 64), (200, 300, 7, 11, 128, 128),
                                      (64, 64, 16, 16, 64, 16), (33, 65, 4, 8, 16, 64)]:
        m = (rng.random((-(-n_q // bm), -(-n_kv // bn))) < 0.4).astype(np.int32)
        _check_plan(m, n_q, n_kv, bm, bn, tm, tn)
    # all-zero mask: empty lists
    z = np.zeros((4, 4), dtype=np.int32)
    _check_plan(z, 64, 64, 16, 16, 16, 64)


@pytest.mark.parametrize("cfg", [(16384, 16384, 4, 2048, 128, 128),
                                 (131072, 131072, 4, 4096, 128, 128)])
def test_gpu_plan_full_size_csr_is_mask_nonzeros(cfg):
    """At benchmark sizes (tile == block) the CSR/CSC lists are exactly the
    nonzero pattern of the upstream mask, in order."""
    n_q, n_kv, s, w, bm, bn = cfg
    m = stk.make_streaming_mask(n_q, n_kv, stk.StreamingMaskSpec(s, w), bm, bn, "cuda")
    plan = stk.build_plan(m, n_q, n_kv, bm, bn, bm, bn)
    mn = m.cpu().numpy()
    rows, cols = np.nonzero(mn)
    nnz = int(plan["nnz"].item())
    assert nnz == len(rows)
    assert np.array_equal(plan["col_idx"][:nnz].cpu().numpy(), cols.astype(np.int32))
    cr, cc = np.nonzero(mn.T)
    assert np.array_equal(plan["row_idx"][:nnz].cpu().numpy(), cc.astype(np.int32))
    counts = np.concatenate([[0], np.cumsum(mn.sum(axis=1))])
    assert np.array_equal(plan["row_ptr"].cpu().numpy(), counts.astype(np.int32))
