"""The bounds-checked debug build, libsbfa_debug.so, on odd shapes.

No memory checker can run on the target pool, so the library also ships a
build compiled with SBFA_DEBUG_BOUNDS: every plan offset, list length and
tile index a kernel reads is range-checked on the device, and a value out of
range is recorded in that library's status word (code 3) and clamped, so the
access stays inside its buffer.  These tests run the forward, backward (both
kernel families, with and without grouped K/V heads) and decode of odd shapes
through the debug build's C ABI and require (a) status 0 - no index left its
range - and (b) results bit-identical to the release build on the same
inputs and plans (the checks change nothing on valid input).
"""

from __future__ import annotations

import ctypes
import math
import os

import pytest
import torch

import sbfa_native as native
import sparse_triton_kernel as stk

pytestmark = pytest.mark.gpu
DEV = "cuda"
DEBUG_LIB = os.path.join(os.path.dirname(native.LIB_PATH), "libsbfa_debug.so")


@pytest.fixture(scope="module")
def dbg():
    if not os.path.exists(DEBUG_LIB):
        pytest.fail("libsbfa_debug.so is not built (run __graft_entry__.build())")
    h = ctypes.CDLL(DEBUG_LIB)
    for name, (args, res) in native._SIGNATURES.items():
        fn = getattr(h, name)
        fn.argtypes = args
        fn.restype = res
    return h


def _status(h) -> int:
    out = ctypes.c_int(0)
    assert h.sbfa_device_status(ctypes.byref(out)) == 0
    return out.value


def _strides(*ts):
    return stk._stride_array(*ts)


def _fwd_bwd(h, q, k, v, do, mask, bm, bn, causal, s, w):
    """Forward and backward through library h with the bridge's plans."""
    B, H, n_q, D = q.shape
    n_kv, hk = k.shape[2], k.shape[1]
    code = native.dtype_code(q.dtype)
    scale = 1.0 / math.sqrt(D)
    p0 = stk._plan_for(mask, 0, q.dtype, D, n_q, n_kv, bm, bn)
    p1 = stk._plan_for(mask, 1, q.dtype, D, n_q, n_kv, bm, bn)
    p2 = stk._plan_for(mask, 2, q.dtype, D, n_q, n_kv, bm, bn)
    o = torch.empty_like(q)
    lse = torch.empty(B, H, n_q, dtype=torch.float32, device=DEV)
    st = native.stream_ptr(q.device)
    assert h.sbfa_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), B, H,
                      n_q, n_kv, D, code, scale, int(causal), s, w, mask.data_ptr(), bm, bn,
                      p0["row_ptr"].data_ptr(), p0["col_idx"].data_ptr(), _strides(q, k, v, o),
                      hk, st) == 0
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    delta = torch.empty(B, H, n_q, dtype=torch.float32, device=DEV)
    ws_bytes = int(h.sbfa_bwd_workspace_bytes(B, H, D, code, hk))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=DEV)
    # stored-dS path (dQ as a GEMM over the dK/dV pass's dS tiles) where it applies
    nnz = stk._plan_nnz(p1)
    ds_bytes = int(h.sbfa_bwd_ds_workspace_bytes(B, H, D, code, nnz)) if p1 is p2 else 0
    ds = torch.empty(max(ds_bytes, 16), dtype=torch.uint8, device=DEV)
    csc = torch.empty_like(p1["col_idx"])
    if ds_bytes:
        assert h.sbfa_plan_csc_positions(p1["row_ptr"].data_ptr(), p1["col_idx"].data_ptr(),
                                         p1["col_ptr"].data_ptr(), p1["row_idx"].data_ptr(),
                                         p1["row_ptr"].numel() - 1, csc.data_ptr(), st) == 0
    assert h.sbfa_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                      do.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                      delta.data_ptr(), B, H, n_q, n_kv, D, code, scale, int(causal), s, w,
                      mask.data_ptr(), bm, bn, p1["row_ptr"].data_ptr(),
                      p1["col_idx"].data_ptr(), p2["col_ptr"].data_ptr(),
                      p2["row_idx"].data_ptr(), _strides(q, k, v, o, do, dq, dk, dv), hk,
                      ws.data_ptr() if ws_bytes else None, ws_bytes,
                      csc.data_ptr() if ds_bytes else None, nnz if ds_bytes else 0,
                      ds.data_ptr() if ds_bytes else None, ds_bytes, st) == 0
    torch.cuda.synchronize()
    return o, lse, dq, dk, dv


# B, H, H_kv, n_q, n_kv, D, bm, bn, causal, S, W, dtype
SHAPES = [
    (1, 2, 2, 1000, 1000, 128, 64, 64, True, 4, 128, torch.bfloat16),    # tensor cores, ragged
    (1, 2, 2, 1023, 1025, 64, 64, 64, True, 4, 200, torch.float16),
    (1, 4, 1, 515, 515, 128, 128, 128, True, 4, 128, torch.bfloat16),    # grouped, split sink tile
    (1, 2, 2, 3, 1025, 128, 16, 64, True, 8, 64, torch.float16),         # n_q < S
    (2, 1, 1, 1025, 1025, 32, 64, 64, True, 4, 128, torch.float32),      # CUDA-core kernels
    (1, 2, 2, 300, 700, 16, 32, 64, False, 0, 0, torch.float16),         # custom mask, generic
]


@pytest.mark.parametrize("shape", SHAPES)
def test_debug_build_is_clean_and_bit_identical(dbg, shape):
    B, H, hk, n_q, n_kv, D, bm, bn, causal, s, w, dt = shape
    g = torch.Generator(device=DEV).manual_seed(7)
    q = torch.randn(B, H, n_q, D, generator=g, device=DEV, dtype=dt)
    k = torch.randn(B, hk, n_kv, D, generator=g, device=DEV, dtype=dt)
    v = torch.randn(B, hk, n_kv, D, generator=g, device=DEV, dtype=dt)
    do = torch.randn(B, H, n_q, D, generator=g, device=DEV, dtype=dt)
    if causal:
        mask = stk.make_streaming_mask(n_q, n_kv, stk.StreamingMaskSpec(s, w), bm, bn, DEV)
    else:
        mask = (torch.rand(-(-n_q // bm), -(-n_kv // bn), generator=g, device=DEV) < 0.5).int()
    _status(dbg)
    got = _fwd_bwd(dbg, q, k, v, do, mask, bm, bn, causal, s, w)
    assert _status(dbg) == 0, "a debug-build kernel found an index out of range"
    want = _fwd_bwd(native.lib(), q, k, v, do, mask, bm, bn, causal, s, w)
    assert native.device_status() == 0
    for nm, a, b in zip(("O", "LSE", "dQ", "dK", "dV"), got, want):
        assert torch.equal(a, b), nm


@pytest.mark.parametrize("B,H,n_kv,D,dt", [(2, 3, 1025, 128, torch.float16),
                                           (4, 8, 100001, 64, torch.bfloat16),
                                           (1, 2, 70, 32, torch.float32)])
def test_debug_build_decode(dbg, B, H, n_kv, D, dt):
    S, W, bn = 4, 2048, 64
    g = torch.Generator(device=DEV).manual_seed(9)
    q = torch.randn(B, H, 1, D, generator=g, device=DEV, dtype=dt)
    k = torch.randn(B, H, n_kv, D, generator=g, device=DEV, dtype=dt)
    v = torch.randn(B, H, n_kv, D, generator=g, device=DEV, dtype=dt)
    mask = stk.make_streaming_mask(1, n_kv, stk.StreamingMaskSpec(S, W), 1, bn, DEV)
    plan = stk._plan_for(mask, 3, dt, D, 1, n_kv, 1, bn)
    outs = []
    for h in (dbg, native.lib()):
        ws = torch.empty(max(16, int(h.sbfa_decode_workspace_bytes(B, H, n_kv, D, bn))),
                         dtype=torch.uint8, device=DEV)
        o = torch.empty_like(q)
        lse = torch.empty(B * H, dtype=torch.float32, device=DEV)
        assert h.sbfa_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                             lse.data_ptr(), B, H, n_kv, D, native.dtype_code(dt),
                             1 / math.sqrt(D), 1, S, W, mask.data_ptr(), 1, bn,
                             plan["row_ptr"].data_ptr(), plan["col_idx"].data_ptr(),
                             ws.data_ptr(), ws.numel(), H, native.stream_ptr(q.device)) == 0
        torch.cuda.synchronize()
        outs.append((o, lse))
    assert _status(dbg) == 0
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
