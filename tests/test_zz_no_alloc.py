"""The allocation-free decode entry point (sbfa_decode_noalloc).

It exists for callers that may not allocate device memory around a decode
step (a serving loop with a fixed, pre-reserved memory budget; a C FFI host
without a device allocator): they hand over only inputs and outputs, and
libsbfa keeps the plan and split partials in its own static device array.
This file is collected last so that, when it fails, a run stopping at the
first failure has already run every other test.  It calls the C ABI
directly and compares against sbfa_decode (the entry point whose caller
provides the workspace) on two calls in a row.
"""

from __future__ import annotations

import math

import pytest
import torch

import sbfa_native as native
import sparse_triton_kernel as stk

pytestmark = pytest.mark.gpu


def _ref_decode(q, k, v, mask, B, H, n_kv, D, code, scale, S, W, bn):
    """The same step through sbfa_decode, with its plan and workspace
    allocated here by the caller."""
    L = native.lib()
    plan = stk.build_plan(mask, 1, n_kv, 1, bn, 1, 64)
    ws = torch.empty(max(16, int(L.sbfa_decode_workspace_bytes(B, H, n_kv, D, bn))),
                     dtype=torch.uint8, device="cuda")
    o = torch.empty_like(q)
    lse = torch.empty(B * H, dtype=torch.float32, device="cuda")
    native.check(L.sbfa_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                               lse.data_ptr(), B, H, n_kv, D, code, scale, 1, S, W,
                               mask.data_ptr(), 1, bn, plan["row_ptr"].data_ptr(),
                               plan["col_idx"].data_ptr(), ws.data_ptr(), ws.numel(),
                               native.stream_ptr(q.device)), "sbfa_decode")
    return o, lse


@pytest.mark.parametrize("B,H,n_kv,D,dtype", [(4, 8, 5000, 128, torch.float16),
                                               (2, 3, 1025, 64, torch.bfloat16),
                                               (64, 32, 4100, 128, torch.float16)])
def test_noalloc_decode_matches_decode_twice(B, H, n_kv, D, dtype):
    L = native.lib()
    S, W, bn = 4, 2048, 64
    scale = 1.0 / math.sqrt(D)
    code = native.dtype_code(dtype)
    g = torch.Generator(device="cuda").manual_seed(123)
    mask = stk.make_streaming_mask(1, n_kv, stk.StreamingMaskSpec(S, W), 1, bn, "cuda")
    for call in range(2):  # two calls in a row: the shared scratch is reused
        q = torch.randn(B, H, 1, D, generator=g, device="cuda", dtype=dtype)
        k = torch.randn(B, H, n_kv, D, generator=g, device="cuda", dtype=dtype)
        v = torch.randn(B, H, n_kv, D, generator=g, device="cuda", dtype=dtype)
        o = torch.full_like(q, float("nan"))
        lse = torch.full((B * H,), float("nan"), dtype=torch.float32, device="cuda")
        native.check(L.sbfa_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                           lse.data_ptr(), B, H, n_kv, D, code, scale, 1, S, W,
                                           mask.data_ptr(), 1, bn,
                                           native.stream_ptr(q.device)), "sbfa_decode_noalloc")
        ro, rlse = _ref_decode(q, k, v, mask, B, H, n_kv, D, code, scale, S, W, bn)
        torch.cuda.synchronize()
        assert torch.isfinite(o).all(), f"call {call}"
        assert torch.allclose(o.float(), ro.float(), atol=2e-2, rtol=2e-2), f"call {call}"
        assert torch.allclose(lse, rlse, atol=1e-4, rtol=1e-4), f"call {call}"


def test_noalloc_rejects_oversize_request():
    """A shape whose plan and partials exceed the static buffer is refused
    with a clear error, before anything is launched."""
    L = native.lib()
    x = torch.empty(16, dtype=torch.float16, device="cuda")
    mask = torch.ones(1, 1, dtype=torch.int32, device="cuda")
    rc = L.sbfa_decode_noalloc(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), None,
                               1, 1, 1 << 30, 128, native.F16, 0.1, 0, 0, 0, mask.data_ptr(), 1,
                               64, native.stream_ptr(x.device))
    assert rc == 1
    assert "static" in native.last_error() and "sbfa_decode" in native.last_error()
