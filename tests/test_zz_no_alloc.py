"""The allocation-free decode entry point (sbfa_decode_noalloc).

It exists for callers that may not allocate device memory around a decode
step: a serving loop that reserved its whole memory budget up front and may
not call cudaMalloc (or grow a caching allocator) per token, and a host that
embeds libsbfa through a plain C FFI with no device allocator of its own.
They hand over only inputs and outputs; libsbfa keeps the decode plan and the
split-KV partials in its own static device array.

This file is collected last so that, when it fails, a run stopping at the
first failure has already run every other test.  It calls the C ABI
directly and compares against sbfa_decode, the entry point whose caller
provides the plan and workspace: the same kernels with the same split count
on the same inputs, so the outputs must match bit for bit.  Consecutive
calls change the sequence length, window and mask, so a plan or partials
left over from the previous call would show up as a mismatch.
"""

from __future__ import annotations

import math

import pytest
import torch

import sbfa_native as native
import sparse_triton_kernel as stk
from oracle import streaming_oracle as orc
from tests.parity import check_half

pytestmark = pytest.mark.gpu


def _ref_decode(q, k, v, mask, B, H, n_kv, D, code, scale, causal, S, W, bn):
    """The same step through sbfa_decode, with its plan and workspace
    allocated here by the caller."""
    L = native.lib()
    plan = stk.build_plan(mask, 1, n_kv, 1, bn, 1, 64)
    ws = torch.empty(max(16, int(L.sbfa_decode_workspace_bytes(B, H, n_kv, D, bn))),
                     dtype=torch.uint8, device="cuda")
    o = torch.full_like(q, float("nan"))
    lse = torch.full((B * H,), float("nan"), dtype=torch.float32, device="cuda")
    native.check(L.sbfa_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                               lse.data_ptr(), B, H, n_kv, D, code, scale, causal, S, W,
                               mask.data_ptr(), 1, bn, plan["row_ptr"].data_ptr(),
                               plan["col_idx"].data_ptr(), ws.data_ptr(), ws.numel(), H,
                               native.stream_ptr(q.device)), "sbfa_decode")
    return o, lse


def _noalloc(q, k, v, mask, B, H, n_kv, D, code, scale, causal, S, W, bn):
    L = native.lib()
    o = torch.full_like(q, float("nan"))
    lse = torch.full((B * H,), float("nan"), dtype=torch.float32, device="cuda")
    native.check(L.sbfa_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                       lse.data_ptr(), B, H, n_kv, D, code, scale, causal, S, W,
                                       mask.data_ptr(), 1, bn, native.stream_ptr(q.device)),
                 "sbfa_decode_noalloc")
    return o, lse


# Each case is two consecutive calls that differ in sequence length, window
# and mask (streaming, then a random custom mask without the token rule), so
# the kept tiles and the split count change between them.
CASES = [
    (4, 8, 128, torch.float16, [(5000, 2048, "stream"), (1500, 512, "random")]),
    (2, 3, 64, torch.bfloat16, [(1025, 256, "random"), (4097, 1024, "stream")]),
    (64, 32, 128, torch.float16, [(4100, 2048, "stream"), (700, 64, "stream")]),
]


@pytest.mark.parametrize("B,H,D,dtype,calls", CASES)
def test_noalloc_decode_matches_decode_on_consecutive_calls(B, H, D, dtype, calls):
    S, bn = 4, 64
    scale = 1.0 / math.sqrt(D)
    code = native.dtype_code(dtype)
    g = torch.Generator(device="cuda").manual_seed(123)
    for call, (n_kv, W, kind) in enumerate(calls):
        if kind == "stream":
            mask = stk.make_streaming_mask(1, n_kv, stk.StreamingMaskSpec(S, W), 1, bn, "cuda")
            causal = 1
        else:
            n_kb = (n_kv + bn - 1) // bn
            mask = (torch.rand(1, n_kb, generator=g, device="cuda") < 0.4).int()
            mask[0, 0] = 1
            causal = 0
        q = torch.randn(B, H, 1, D, generator=g, device="cuda", dtype=dtype)
        k = torch.randn(B, H, n_kv, D, generator=g, device="cuda", dtype=dtype)
        v = torch.randn(B, H, n_kv, D, generator=g, device="cuda", dtype=dtype)
        o, lse = _noalloc(q, k, v, mask, B, H, n_kv, D, code, scale, causal, S, W, bn)
        ro, rlse = _ref_decode(q, k, v, mask, B, H, n_kv, D, code, scale, causal, S, W, bn)
        torch.cuda.synchronize()
        assert torch.equal(o, ro), f"call {call}: O differs from sbfa_decode"
        assert torch.equal(lse, rlse), f"call {call}: LSE differs from sbfa_decode"
        # and against the float64 oracle on two heads
        for b, h in ((0, 0), (B - 1, H - 1)):
            if kind == "stream":
                ref, _ = orc.streaming_rows_forward(q[b, h], k[b, h], v[b, h], [0], S, W, scale)
            else:
                ref = orc.attention_forward(q[b:b + 1, h:h + 1].double().cpu(),
                                            k[b:b + 1, h:h + 1].double().cpu(),
                                            v[b:b + 1, h:h + 1].double().cpu(), mask.cpu(),
                                            block_m=1, block_n=bn, is_causal=False,
                                            sink_size=0, window_size=0)[0, 0]
            check_half(o[b, h], ref, dtype, f"noalloc call {call} b{b} h{h}")
    assert native.device_status() == 0


def test_noalloc_rejects_oversize_request():
    """A shape whose plan and partials exceed the static buffer is refused
    with a clear error, before anything is launched."""
    L = native.lib()
    x = torch.empty(16, dtype=torch.float16, device="cuda")
    mask = torch.ones(1, 1, dtype=torch.int32, device="cuda")
    before = native.launch_count()
    rc = L.sbfa_decode_noalloc(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), None,
                               1, 1, 1 << 30, 128, native.F16, 0.1, 0, 0, 0, mask.data_ptr(), 1,
                               64, native.stream_ptr(x.device))
    assert rc == 1
    assert "static" in native.last_error() and "sbfa_decode" in native.last_error()
    assert native.launch_count() == before


def test_noalloc_rejects_bad_arguments_before_any_launch():
    """Invalid tensors or shapes are refused with sbfa_decode's own checks
    before the plan kernels run, so a refused call never touches the shared
    scratch of a caller's earlier, valid calls."""
    L = native.lib()
    x = torch.empty(4096, dtype=torch.float16, device="cuda")
    mask = torch.ones(1, 16, dtype=torch.int32, device="cuda")
    s = native.stream_ptr(x.device)
    before = native.launch_count()
    bad = [
        (None, x.data_ptr(), 128, native.F16),            # NULL q
        (x.data_ptr() + 2, x.data_ptr(), 128, native.F16),  # misaligned q
        (x.data_ptr(), x.data_ptr(), 96, native.F64),     # no decode kernel for float64
        (x.data_ptr(), x.data_ptr(), 0, native.F16),      # bad head_dim
    ]
    for qp, kp, D, code in bad:
        rc = L.sbfa_decode_noalloc(qp, kp, kp, kp, None, 1, 1, 1000, D, code, 0.1, 1, 4, 64,
                                   mask.data_ptr(), 1, 64, s)
        assert rc != 0
    assert native.launch_count() == before
