"""Forward / backward / decode parity of libsbfa against the oracle.

Tolerances (written per dtype, from the upstream verification protocol
and the north-star bar):
  * float64: forward 1e-9; gradients 1e-6 (the backward reads the fp32 LSE
    and Delta the upstream format stores, sparse_triton_kernel.py:653,716);
  * float32: forward atol = rtol = 1e-4 (benchmark.py:166-195), gradients
    atol = rtol = 1e-3 (benchmark.py:322-355);
  * float16 / bfloat16: max-abs <= 2e-2 and rel-L2 <= 5e-3 (fixed bounds,
    tests/parity.py) against a float64 oracle on the same (rounded) inputs.
"""

from __future__ import annotations

import math
import os

import numpy as np
import pytest
import torch

import sbfa_native as native
import sparse_triton_kernel as stk
from oracle import streaming_oracle as orc
from tests.golden.make_golden import ATTN_CASES, ATTN_TC_CASES
from tests.parity import check_half

pytestmark = pytest.mark.gpu

DEV = "cuda"


def close(got: torch.Tensor, ref: torch.Tensor, dtype: torch.dtype, kind: str = "fwd",
          label: str = ""):
    got = got.double().cpu()
    ref = ref.double().cpu()
    assert torch.isfinite(got).all(), "non-finite output"
    if dtype == torch.float64:
        tol = 1e-9 if kind == "fwd" else 1e-6
        assert torch.allclose(got, ref, atol=tol, rtol=tol), (got - ref).abs().max()
    elif dtype == torch.float32:
        tol = 1e-4 if kind == "fwd" else 1e-3
        assert torch.allclose(got, ref, atol=tol, rtol=tol), (got - ref).abs().max()
    else:
        check_half(got, ref, dtype, label or kind)


def run(q, k, v, mask, bm, bn, causal, s, w, do=None, scale=None):
    q = q.detach().clone().requires_grad_(do is not None)
    k = k.detach().clone().requires_grad_(do is not None)
    v = v.detach().clone().requires_grad_(do is not None)
    o = stk.block_sparse_attention(q, k, v, mask, softmax_scale=scale, block_m=bm, block_n=bn,
                                   is_causal=causal, sink_size=s, window_size=w)
    if do is None:
        return o.detach(), None, None, None
    o.backward(do)
    return o.detach(), q.grad, k.grad, v.grad


@pytest.fixture(scope="module")
def golden(golden_dir):
    return np.load(os.path.join(golden_dir, "attention_cases.npz"))


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("name", [c[0] for c in ATTN_CASES])
def test_golden_cases(golden, name, dtype):
    """Every stored upstream case, forward and gradients, in every dtype."""
    p = f"{name}__"
    B, H, n_q, n_kv, D, bm, bn, causal, s, w = golden[p + "params"].tolist()
    t = {x: torch.from_numpy(golden[p + x]) for x in ("q", "k", "v", "do")}
    mask = torch.from_numpy(golden[p + "mask"]).to(DEV)
    qd, kd, vd, dod = (t[x].to(DEV, dtype) for x in ("q", "k", "v", "do"))
    o, dq, dk, dv = run(qd, kd, vd, mask, bm, bn, bool(causal), s, w, do=dod)
    if dtype == torch.float64:
        refs = {x: torch.from_numpy(golden[p + x]) for x in ("o", "dq", "dk", "dv")}
    else:  # oracle on the rounded inputs
        ro, rdq, rdk, rdv = orc.attention_forward_backward(
            qd.double().cpu(), kd.double().cpu(), vd.double().cpu(), dod.double().cpu(),
            golden[p + "mask"], block_m=bm, block_n=bn, is_causal=bool(causal), sink_size=s,
            window_size=w)
        refs = {"o": ro, "dq": rdq, "dk": rdk, "dv": rdv}
    close(o, refs["o"], dtype, "fwd")
    close(dq, refs["dq"], dtype, "bwd")
    close(dk, refs["dk"], dtype, "bwd")
    close(dv, refs["dv"], dtype, "bwd")


@pytest.mark.parametrize("dq_path", ["stored", "recompute"])
@pytest.mark.parametrize("name", [c[0] for c in ATTN_TC_CASES])
def test_tensor_core_golden_cases(golden_dir, monkeypatch, name, dq_path):
    """Upstream outputs at the tensor-core shapes (16-bit inputs, head_dim
    128 / 64, 128 x 128 blocks), produced by the reference itself: the
    tcgen05 forward, dK/dV and both dQ kernels (the GEMM over stored dS at
    head_dim 128, the recomputing pass) against them directly."""
    from tests.test_oracle_golden import tc_case_inputs
    g = np.load(os.path.join(golden_dir, "attention_tc_cases.npz"))
    (B, H, n_q, n_kv, D, bm, bn, causal, s, w), dt, mask, ins, outs = tc_case_inputs(g, name)
    if dq_path == "stored" and D != 128:
        pytest.skip("dS is stored for the dQ GEMM at head_dim 128 only")
    if dq_path == "recompute":
        monkeypatch.setenv(stk.DS_BUDGET_ENV, "0")
    else:
        monkeypatch.delenv(stk.DS_BUDGET_ENV, raising=False)
    want_dq = "dq_gemm_kernel" if dq_path == "stored" else "dq_tc_kernel"
    qd, kd, vd, dod = (ins[x].to(DEV) for x in ("q", "k", "v", "do"))
    native.timing_read()
    native.timing(True)
    try:
        o, dq, dk, dv = run(qd, kd, vd, torch.from_numpy(mask).to(DEV), bm, bn, bool(causal),
                            s, w, do=dod)
        ran = native.timing_read()
    finally:
        native.timing(False)
    assert {"fwd_tc_kernel", "dkdv_tc_kernel", want_dq} <= set(ran), ran
    for nm, got in (("O", o), ("dQ", dq), ("dK", dk), ("dV", dv)):
        check_half(got, outs[nm.lower()], dt, f"{name} {nm}")
    assert native.device_status() == 0


SHAPES = [
    # B, H, n_q, n_kv, D, bm, bn, causal, S, W
    (1, 4, 1024, 1024, 64, 64, 64, True, 4, 256),     # cfg1 geometry
    (2, 2, 512, 512, 128, 128, 128, True, 4, 128),
    (1, 2, 300, 700, 128, 64, 128, True, 4, 200),     # bottom-right, ragged
    (1, 2, 256, 256, 64, 128, 64, True, 0, 100),      # window only
    (1, 1, 129, 257, 128, 128, 128, True, 1, 64),
    (1, 2, 256, 256, 128, 64, 64, False, 0, 0),       # dense non-causal
    (1, 2, 200, 384, 32, 16, 32, True, 8, 40),
]


def _inputs(B, H, n_q, n_kv, D, dtype, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = torch.randn(B, H, n_q, D, generator=g, device=DEV, dtype=dtype)
    k = torch.randn(B, H, n_kv, D, generator=g, device=DEV, dtype=dtype)
    v = torch.randn(B, H, n_kv, D, generator=g, device=DEV, dtype=dtype)
    g1 = torch.Generator(device=DEV).manual_seed(1)
    do = torch.randn(B, H, n_q, D, generator=g1, device=DEV, dtype=dtype)
    return q, k, v, do


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", SHAPES)
def test_streaming_shapes(shape, dtype):
    B, H, n_q, n_kv, D, bm, bn, causal, s, w = shape
    q, k, v, do = _inputs(B, H, n_q, n_kv, D, dtype)
    if causal:
        mask = stk.make_streaming_mask(n_q, n_kv, stk.StreamingMaskSpec(s, w), bm, bn, DEV)
    else:
        mask = stk.make_dense_mask(n_q, n_kv, bm, bn, device=DEV) if (
            n_q % bm == 0 and n_kv % bn == 0) else torch.ones(
            -(-n_q // bm), -(-n_kv // bn), dtype=torch.int32, device=DEV)
    o, dq, dk, dv = run(q, k, v, mask, bm, bn, causal, s, w, do=do)
    ro, rdq, rdk, rdv = orc.attention_forward_backward(
        q.double().cpu(), k.double().cpu(), v.double().cpu(), do.double().cpu(), mask.cpu(),
        block_m=bm, block_n=bn, is_causal=causal, sink_size=s, window_size=w)
    close(o, ro, dtype, "fwd")
    close(dq, rdq, dtype, "bwd")
    close(dk, rdk, dtype, "bwd")
    close(dv, rdv, dtype, "bwd")
    assert native.device_status() == 0


def test_custom_mask_causal_and_not():
    torch.manual_seed(0)
    for causal in (False, True):
        q, k, v, do = _inputs(1, 2, 192, 320, 64, torch.bfloat16, seed=3)
        mask = (torch.rand(6, 10, device=DEV) < 0.5).int()
        o, dq, dk, dv = run(q, k, v, mask, 32, 32, causal, 4, 48, do=do)
        ro, rdq, rdk, rdv = orc.attention_forward_backward(
            q.double().cpu(), k.double().cpu(), v.double().cpu(), do.double().cpu(), mask.cpu(),
            block_m=32, block_n=32, is_causal=causal, sink_size=4, window_size=48)
        for a, b, kind in ((o, ro, "fwd"), (dq, rdq, "bwd"), (dk, rdk, "bwd"), (dv, rdv, "bwd")):
            close(a, b, torch.bfloat16, kind)


def test_fully_masked_rows_give_zero_and_finite_grads():
    """Upstream tests/test_fully_masked_row.py:134-175 on this kernel."""
    B, H, N, D, bm = 1, 2, 32, 16, 16
    q = torch.randn(B, H, N, D, device=DEV, requires_grad=True)
    k = torch.randn(B, H, N, D, device=DEV, requires_grad=True)
    v = torch.randn(B, H, N, D, device=DEV, requires_grad=True)
    mask = torch.zeros((2, 2), dtype=torch.int32, device=DEV)
    mask[1, 1] = 1
    out = stk.block_sparse_attention(q, k, v, mask, block_m=bm, block_n=bm, is_causal=False)
    assert torch.isfinite(out).all()
    assert torch.equal(out[:, :, :bm], torch.zeros_like(out[:, :, :bm]))
    out.backward(torch.randn_like(out))
    for g in (q.grad, k.grad, v.grad):
        assert g is not None and torch.isfinite(g).all()
    assert torch.equal(q.grad[:, :, :bm], torch.zeros_like(q.grad[:, :, :bm]))


def test_gradcheck_float64():
    """Finite differences vs the analytic backward (upstream benchmark.py:203-270
    fp64 tier: eps 1e-6, atol 1e-5, rtol 1e-3)."""
    B, H, N, D, bm = 1, 2, 64, 16, 16
    g = torch.Generator(device=DEV).manual_seed(0)
    q, k, v = (torch.randn(B, H, N, D, generator=g, device=DEV, dtype=torch.float64,
                           requires_grad=True) for _ in range(3))
    mask = stk.make_streaming_mask(N, N, stk.StreamingMaskSpec(4, 16), bm, bm, DEV)

    def fn(a, b, c):
        return stk.block_sparse_attention(a, b, c, mask, softmax_scale=1 / math.sqrt(D),
                                          block_m=bm, block_n=bm, is_causal=True,
                                          sink_size=4, window_size=16)

    assert torch.autograd.gradcheck(fn, (q, k, v), eps=1e-6, atol=1e-5, rtol=1e-3,
                                    fast_mode=False)


DECODE = [
    # B, H, n_kv, D, bn, S, W, dtype
    (4, 8, 1000, 128, 64, 4, 256, torch.float16),
    (2, 4, 1023, 128, 64, 4, 256, torch.bfloat16),
    (2, 4, 1025, 64, 64, 4, 256, torch.float16),
    (1, 2, 5000, 128, 64, 0, 2048, torch.float32),
    (3, 2, 777, 16, 32, 8, 0, torch.float16),       # sink only
    (2, 2, 300, 128, 64, 4, 4096, torch.bfloat16),  # window covers all
    (64, 8, 4100, 128, 64, 4, 2048, torch.float16), # many heads, several splits
]


@pytest.mark.parametrize("case", DECODE)
def test_decode_matches_oracle(case):
    B, H, n_kv, D, bn, s, w, dtype = case
    q, k, v, _ = _inputs(B, H, 1, n_kv, D, dtype, seed=5)
    mask = stk.make_streaming_mask(1, n_kv, stk.StreamingMaskSpec(s, w), 1, bn, DEV)
    before = native.launch_count()
    o, *_ = run(q, k, v, mask, 1, bn, True, s, w)
    assert native.launch_count() > before
    scale = 1 / math.sqrt(D)
    for b in range(B):
        for h in range(H):
            ro, _ = orc.streaming_rows_forward(q[b, h], k[b, h], v[b, h], [0], s, w, scale)
            if dtype == torch.float32:
                assert torch.allclose(o[b, h].double(), ro, atol=1e-4, rtol=1e-4)
            else:
                check_half(o[b, h], ro, dtype, f"decode b{b} h{h}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("H,Hkv,n_kv,D", [(8, 2, 3000, 128), (8, 1, 2500, 128),
                                          (6, 2, 1777, 64), (32, 4, 4100, 128),
                                          (32, 1, 1500, 128), (20, 1, 700, 64),
                                          (4, 2, 50, 128)])
def test_grouped_query_decode(dtype, H, Hkv, n_kv, D):
    """N_Q = 1 with fewer K/V heads than query heads runs the tensor-core
    grouped decode kernel (each K/V row read once for up to 16 query heads
    of its group; groups of 2, 3, 4, 8, 20 (two CTAs of 10) and 32 (two of
    16); a 50-key cache in one tile, hence one split), against the float64
    oracle per query head."""
    B, S, W = 2, 4, 1024
    g = torch.Generator(device=DEV).manual_seed(31)
    q = torch.randn(B, H, 1, D, generator=g, device=DEV, dtype=dtype)
    k = torch.randn(B, Hkv, n_kv, D, generator=g, device=DEV, dtype=dtype)
    v = torch.randn(B, Hkv, n_kv, D, generator=g, device=DEV, dtype=dtype)
    mask = stk.make_streaming_mask(1, n_kv, stk.StreamingMaskSpec(S, W), 1, 64, DEV)
    native.timing_read()
    native.timing(True)
    try:
        with torch.no_grad():
            o = stk.block_sparse_attention(q, k, v, mask, block_m=1, block_n=64, is_causal=True,
                                           sink_size=S, window_size=W)
        ran = native.timing_read()
    finally:
        native.timing(False)
    assert "decode_gqa_kernel" in ran, ran
    assert "decode_split_kernel" not in ran and not any(n.startswith("fwd") for n in ran), ran
    scale = 1 / math.sqrt(D)
    grp = H // Hkv
    for b in range(B):
        for h in range(H):
            ro, _ = orc.streaming_rows_forward(q[b, h], k[b, h // grp], v[b, h // grp], [0], S,
                                               W, scale)
            check_half(o[b, h], ro, dtype, f"gqa decode b{b} h{h}")
    assert native.device_status() == 0


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 64)])
def test_grouped_query_backward_splits_the_sink_tile(monkeypatch, dtype, D):
    """With grouped K/V heads the first key tile is seen by every query tile
    of every query head of its group.  Its dK/dV work is split over one CTA
    per query head (fp32 partials, summed by a second kernel); the result
    matches the oracle and the unsplit single-CTA path."""
    B, H, Hkv, N, S, W = 1, 8, 1, 2048, 4, 256
    q, k, v, do = (torch.randn(B, h, N, D, generator=torch.Generator(device=DEV).manual_seed(s),
                               device=DEV, dtype=dtype)
                   for s, h in ((1, H), (2, Hkv), (3, Hkv), (4, H)))
    mask = stk.make_streaming_mask(N, N, stk.StreamingMaskSpec(S, W), 128, 128, DEV)
    L = native.lib()
    assert L.sbfa_bwd_workspace_bytes(B, H, D, native.dtype_code(dtype), Hkv) > 0
    native.timing_read()
    native.timing(True)
    try:
        o, dq, dk, dv = run(q, k, v, mask, 128, 128, True, S, W, do=do)
        ran = native.timing_read()
    finally:
        native.timing(False)
    assert "dkdv_sink_reduce_kernel" in ran, ran
    # the same call without split scratch: one CTA per unit streams every head
    monkeypatch.setattr(L, "sbfa_bwd_workspace_bytes", lambda *a: 0)
    _, dq1, dk1, dv1 = run(q, k, v, mask, 128, 128, True, S, W, do=do)
    monkeypatch.undo()
    assert torch.equal(dq, dq1)            # the dQ kernel is untouched
    for a, b, nm in ((dk, dk1, "dK"), (dv, dv1, "dV")):
        check_half(a, b.double(), dtype, f"split vs unsplit {nm}")
    # against the oracle: K/V expanded to every query head, gradients summed
    # over each group
    kx, vx = (t.expand(B, H, N, D) for t in (k, v))
    ro, rdq, rdk, rdv = orc.attention_forward_backward(
        q.double().cpu(), kx.double().cpu(), vx.double().cpu(), do.double().cpu(), mask.cpu(),
        block_m=128, block_n=128, is_causal=True, sink_size=S, window_size=W)
    check_half(o, ro, dtype, "O")
    check_half(dq, rdq, dtype, "dQ")
    check_half(dk, rdk.sum(dim=1, keepdim=True), dtype, "dK")
    check_half(dv, rdv.sum(dim=1, keepdim=True), dtype, "dV")
    assert native.device_status() == 0


def test_decode_custom_mask_and_noncausal():
    q, k, v, _ = _inputs(2, 3, 1, 640, 128, torch.float16, seed=7)
    mask = (torch.rand(1, 10, device=DEV) < 0.5).int()
    mask[0, 3] = 1
    for causal in (False, True):
        o, *_ = run(q, k, v, mask, 1, 64, causal, 4, 100)
        ro = orc.attention_forward(q.double().cpu(), k.double().cpu(), v.double().cpu(),
                                   mask.cpu(), block_m=1, block_n=64, is_causal=causal,
                                   sink_size=4, window_size=100)
        close(o, ro, torch.float16)


@pytest.mark.parametrize("dtype,D,H,Hkv,bn", [(torch.bfloat16, 128, 8, 2, 32),
                                              (torch.float16, 64, 12, 3, 64)])
def test_grouped_query_decode_custom_mask_and_grad(dtype, D, H, Hkv, bn):
    """The tensor-core grouped decode under a random block mask (with 32-key
    mask blocks the 64-key decode tiles are partly kept), causal and not,
    against the oracle on K/V repeated per group; with gradients, its LSE
    feeds the backward, checked the same way."""
    B, n_kv, S, W = 2, 777, 4, 200
    gen = torch.Generator(device=DEV).manual_seed(41)
    q = torch.randn(B, H, 1, D, generator=gen, device=DEV, dtype=dtype)
    k = torch.randn(B, Hkv, n_kv, D, generator=gen, device=DEV, dtype=dtype)
    v = torch.randn(B, Hkv, n_kv, D, generator=gen, device=DEV, dtype=dtype)
    do = torch.randn(B, H, 1, D, generator=gen, device=DEV, dtype=dtype)
    n_kb = (n_kv + bn - 1) // bn
    mask = (torch.rand(1, n_kb, generator=gen, device=DEV) < 0.5).int()
    mask[0, 0] = mask[0, -1] = 1
    rep = H // Hkv
    ke, ve = (t.repeat_interleave(rep, dim=1) for t in (k, v))
    for causal in (False, True):
        native.timing_read()
        native.timing(True)
        try:
            o, dq, dk, dv = run(q, k, v, mask, 1, bn, causal, S, W, do=do)
            ran = native.timing_read()
        finally:
            native.timing(False)
        assert "decode_gqa_kernel" in ran, ran
        ro, rdq, rdk, rdv = orc.attention_forward_backward(
            q.double().cpu(), ke.double().cpu(), ve.double().cpu(), do.double().cpu(),
            mask.cpu(), block_m=1, block_n=bn, is_causal=causal, sink_size=S, window_size=W)
        rdk = rdk.view(B, Hkv, rep, n_kv, D).sum(2)
        rdv = rdv.view(B, Hkv, rep, n_kv, D).sum(2)
        check_half(o, ro, dtype, f"gqa decode causal={causal} O")
        check_half(dq, rdq, dtype, f"gqa decode causal={causal} dQ")
        check_half(dk, rdk, dtype, f"gqa decode causal={causal} dK")
        check_half(dv, rdv, dtype, f"gqa decode causal={causal} dV")
    # no kept block: every head's output is 0 (upstream's empty-row rule)
    o, *_ = run(q, k, v, torch.zeros_like(mask), 1, bn, False, S, W)
    assert torch.equal(o, torch.zeros_like(o))
    assert native.device_status() == 0


@pytest.mark.parametrize("dtype,H,Hkv", [(torch.bfloat16, 2, 2), (torch.float16, 4, 1)])
def test_stored_ds_dq_matches_recompute(monkeypatch, dtype, H, Hkv):
    """At head_dim 128 the dK/dV pass stores dS and dQ is a GEMM over the
    stored tiles (dq_gemm_kernel); with a zero budget the third pass
    recomputes S, P and dP instead (dq_tc_kernel).  Both match the oracle,
    dK and dV are bit-identical between them (same pass, same arithmetic),
    and dQ agrees to rounding."""
    B, N, S, W, D = 1, 700, 4, 256, 128
    gen = torch.Generator(device=DEV).manual_seed(17)
    q = torch.randn(B, H, N, D, generator=gen, device=DEV, dtype=dtype)
    k = torch.randn(B, Hkv, N, D, generator=gen, device=DEV, dtype=dtype)
    v = torch.randn(B, Hkv, N, D, generator=gen, device=DEV, dtype=dtype)
    do = torch.randn(B, H, N, D, generator=gen, device=DEV, dtype=dtype)
    mask = stk.make_streaming_mask(N, N, stk.StreamingMaskSpec(S, W), 128, 128, DEV)
    outs = {}
    for name, budget in (("stored", None), ("recompute", "0")):
        if budget is None:
            monkeypatch.delenv(stk.DS_BUDGET_ENV, raising=False)
        else:
            monkeypatch.setenv(stk.DS_BUDGET_ENV, budget)
        native.timing_read()
        native.timing(True)
        try:
            outs[name] = run(q, k, v, mask, 128, 128, True, S, W, do=do)
            ran = native.timing_read()
        finally:
            native.timing(False)
        want, other = ("dq_gemm_kernel", "dq_tc_kernel") if budget is None else (
            "dq_tc_kernel", "dq_gemm_kernel")
        assert want in ran and other not in ran, ran
    rep = H // Hkv
    ke, ve = (t.repeat_interleave(rep, dim=1) for t in (k, v))
    ro, rdq, rdk, rdv = orc.attention_forward_backward(
        q.double().cpu(), ke.double().cpu(), ve.double().cpu(), do.double().cpu(), mask.cpu(),
        block_m=128, block_n=128, is_causal=True, sink_size=S, window_size=W)
    rdk = rdk.view(B, Hkv, rep, N, D).sum(2)
    rdv = rdv.view(B, Hkv, rep, N, D).sum(2)
    for name, (o, dq, dk, dv) in outs.items():
        check_half(dq, rdq, dtype, f"{name} dQ")
        check_half(dk, rdk, dtype, f"{name} dK")
        check_half(dv, rdv, dtype, f"{name} dV")
    a, b = outs["stored"], outs["recompute"]
    assert torch.equal(a[0], b[0]) and torch.equal(a[2], b[2]) and torch.equal(a[3], b[3])
    assert (a[1].float() - b[1].float()).abs().max().item() < 2e-2
    assert native.device_status() == 0


def test_decode_backward_runs_generic_path():
    q, k, v, do = _inputs(1, 2, 1, 500, 64, torch.float32, seed=2)
    mask = stk.make_streaming_mask(1, 500, stk.StreamingMaskSpec(4, 128), 1, 64, DEV)
    o, dq, dk, dv = run(q, k, v, mask, 1, 64, True, 4, 128, do=do)
    ro, rdq, rdk, rdv = orc.attention_forward_backward(
        q.double().cpu(), k.double().cpu(), v.double().cpu(), do.double().cpu(), mask.cpu(),
        block_m=1, block_n=64, is_causal=True, sink_size=4, window_size=128)
    close(o, ro, torch.float32)
    close(dq, rdq, torch.float32, "bwd")
    close(dk, rdk, torch.float32, "bwd")
    close(dv, rdv, torch.float32, "bwd")


def test_plan_cache_reused_and_invalidated():
    q, k, v, _ = _inputs(1, 1, 256, 256, 64, torch.float16)
    mask = stk.make_streaming_mask(256, 256, stk.StreamingMaskSpec(4, 64), 64, 64, DEV)
    run(q, k, v, mask, 64, 64, True, 4, 64)
    n0 = native.launch_count()
    run(q, k, v, mask, 64, 64, True, 4, 64)
    steady = native.launch_count() - n0
    mask.zero_()  # in-place edit -> new version -> plan rebuilt
    mask[:, 0] = 1
    n1 = native.launch_count()
    o, *_ = run(q, k, v, mask, 64, 64, True, 4, 64)
    assert native.launch_count() - n1 > steady
    ro = orc.attention_forward(q.double().cpu(), k.double().cpu(), v.double().cpu(), mask.cpu(),
                               block_m=64, block_n=64, is_causal=True, sink_size=4, window_size=64)
    close(o, ro, torch.float16)


def test_errors_are_raised():
    q, k, v, _ = _inputs(1, 1, 64, 64, 16, torch.float32)
    with pytest.raises(ValueError, match="block_mask has shape"):
        stk.block_sparse_attention(q, k, v, torch.ones(3, 3, dtype=torch.int32, device=DEV),
                                   block_m=16, block_n=16)
    with pytest.raises(ValueError, match="K and V must share shape"):
        stk.block_sparse_attention(q, k, v[:, :, :32], torch.ones(4, 4, dtype=torch.int32,
                                   device=DEV), block_m=16, block_n=16)
    with pytest.raises(ValueError, match="unsupported dtype"):
        stk.block_sparse_attention(q.int(), k.int(), v.int(), torch.ones(
            4, 4, dtype=torch.int32, device=DEV), block_m=16, block_n=16)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128])
def test_tensor_core_path_empty_rows(dtype, D):
    """bf16/fp16 with D in {64, 128} runs the tcgen05 forward: a query tile
    with no kept block, rows with no visible key inside kept tiles, and a
    ragged last tile must all match the oracle (zeros where nothing is
    visible)."""
    n_q, n_kv, bm = 384, 300, 128
    q, k, v, do = _inputs(2, 2, n_q, n_kv, D, dtype, seed=9)
    mask = torch.ones(3, 3, dtype=torch.int32, device=DEV)
    mask[0, :] = 0          # first query tile sees nothing
    mask[2, 0] = 0
    for causal in (False, True):
        o, dq, dk, dv = run(q, k, v, mask, bm, bm, causal, 0, 40, do=do)
        ro, rdq, rdk, rdv = orc.attention_forward_backward(
            q.double().cpu(), k.double().cpu(), v.double().cpu(), do.double().cpu(), mask.cpu(),
            block_m=bm, block_n=bm, is_causal=causal, sink_size=0, window_size=40)
        assert torch.equal(o[:, :, :bm].float(), torch.zeros_like(o[:, :, :bm].float()))
        for a, b, kind in ((o, ro, "fwd"), (dq, rdq, "bwd"), (dk, rdk, "bwd"), (dv, rdv, "bwd")):
            close(a, b, dtype, kind)
    assert native.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_more_queries_than_keys_streaming(dtype):
    """n_q > n_kv under the bottom-right alignment: the first n_q - n_kv
    query rows sit at negative positions and see no key under the
    streaming mask, so they are zero with zero dQ; the rest match the
    oracle (tensor-core path for bf16, generic path for fp32)."""
    n_q, n_kv, s, w = 640, 400, 4, 96
    q, k, v, do = _inputs(1, 2, n_q, n_kv, 128, dtype, seed=5)
    mask = stk.make_streaming_mask(n_q, n_kv, stk.StreamingMaskSpec(s, w), 128, 128, DEV)
    o, dq, dk, dv = run(q, k, v, mask, 128, 128, True, s, w, do=do)
    ro, rdq, rdk, rdv = orc.attention_forward_backward(
        q.double().cpu(), k.double().cpu(), v.double().cpu(), do.double().cpu(), mask.cpu(),
        block_m=128, block_n=128, is_causal=True, sink_size=s, window_size=w)
    dead = n_q - n_kv
    assert torch.count_nonzero(o[:, :, :dead]).item() == 0
    assert torch.count_nonzero(dq[:, :, :dead]).item() == 0
    for a, b, kind in ((o, ro, "fwd"), (dq, rdq, "bwd"), (dk, rdk, "bwd"), (dv, rdv, "bwd")):
        close(a, b, dtype, kind)
    assert native.device_status() == 0


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 64),
                                     (torch.float32, 64), (torch.bfloat16, 96)])
def test_strided_views_read_in_place(dtype, D):
    """Q/K/V as transposes of [B, N, H, D] storage (the layout behind
    Llama-style attention) and dO as a transposed view: the kernels read them
    through their strides, with results bit-identical to the contiguous call
    (same data, same arithmetic) and equal to the oracle."""
    B, H, n, S, W, bm = 2, 3, 640, 4, 192, 64
    g = torch.Generator(device=DEV).manual_seed(5)
    base = [torch.randn(B, n, H, D, generator=g, device=DEV, dtype=dtype) for _ in range(4)]
    q, k, v, do = (t.transpose(1, 2) for t in base)
    assert not q.is_contiguous()
    mask = stk.make_streaming_mask(n, n, stk.StreamingMaskSpec(S, W), bm, bm, DEV)
    outs = []
    for qq, kk, vv, gg in ((q, k, v, do), tuple(t.contiguous() for t in (q, k, v, do))):
        qq, kk, vv = (t.detach().requires_grad_(True) for t in (qq, kk, vv))
        o = stk.block_sparse_attention(qq, kk, vv, mask, block_m=bm, block_n=bm, is_causal=True,
                                       sink_size=S, window_size=W)
        o.backward(gg)
        outs.append((o.detach(), qq.grad, kk.grad, vv.grad))
    assert native.device_status() == 0
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    ro, rdq, rdk, rdv = orc.attention_forward_backward(
        q.double().cpu(), k.double().cpu(), v.double().cpu(), do.double().cpu(), mask.cpu(),
        block_m=bm, block_n=bm, is_causal=True, sink_size=S, window_size=W)
    close(outs[0][0], ro, dtype, "fwd")
    for got, ref in zip(outs[0][1:], (rdq, rdk, rdv)):
        close(got, ref, dtype, "bwd")


def test_unaligned_view_falls_back_to_copy():
    """A view whose row stride is not a multiple of 8 elements cannot be read
    by TMA; the bridge copies it (as upstream always does) and the result is
    unchanged."""
    B, H, n, D = 1, 2, 256, 64
    g = torch.Generator(device=DEV).manual_seed(6)
    wide = torch.randn(B, H, n, D + 4, generator=g, device=DEV, dtype=torch.bfloat16)
    q = wide[..., :D]  # row stride D + 4
    k, v = (torch.randn(B, H, n, D, generator=g, device=DEV, dtype=torch.bfloat16)
            for _ in range(2))
    mask = stk.make_streaming_mask(n, n, stk.StreamingMaskSpec(4, 64), 64, 64, DEV)
    kw = dict(block_m=64, block_n=64, is_causal=True, sink_size=4, window_size=64)
    a = stk.block_sparse_attention(q, k, v, mask, **kw)
    b = stk.block_sparse_attention(q.contiguous(), k, v, mask, **kw)
    assert torch.equal(a, b)


@pytest.mark.parametrize("dtype,D,H,Hkv", [(torch.bfloat16, 128, 4, 2), (torch.float16, 64, 6, 1),
                                           (torch.float32, 64, 4, 2), (torch.bfloat16, 64, 3, 3)])
def test_grouped_query_heads(dtype, D, H, Hkv):
    """Grouped-query attention: K/V with H / g heads, query head h reading
    key/value head h // g.  Equal to the oracle run on K/V repeated g times,
    with dK/dV the sums over each group's query heads."""
    B, n, S, W, bm = 2, 384, 4, 128, 64
    g = torch.Generator(device=DEV).manual_seed(9)
    q = torch.randn(B, H, n, D, generator=g, device=DEV, dtype=dtype)
    k = torch.randn(B, Hkv, n, D, generator=g, device=DEV, dtype=dtype)
    v = torch.randn(B, Hkv, n, D, generator=g, device=DEV, dtype=dtype)
    do = torch.randn(B, H, n, D, generator=g, device=DEV, dtype=dtype)
    mask = stk.make_streaming_mask(n, n, stk.StreamingMaskSpec(S, W), bm, bm, DEV)
    qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = stk.block_sparse_attention(qq, kk, vv, mask, block_m=bm, block_n=bm, is_causal=True,
                                   sink_size=S, window_size=W)
    o.backward(do)
    assert native.device_status() == 0
    rep = H // Hkv
    ke, ve = (t.repeat_interleave(rep, dim=1) for t in (k, v))
    ro, rdq, rdk, rdv = orc.attention_forward_backward(
        q.double().cpu(), ke.double().cpu(), ve.double().cpu(), do.double().cpu(), mask.cpu(),
        block_m=bm, block_n=bm, is_causal=True, sink_size=S, window_size=W)
    rdk = rdk.view(B, Hkv, rep, n, D).sum(2)
    rdv = rdv.view(B, Hkv, rep, n, D).sum(2)
    close(o, ro, dtype, "fwd")
    close(qq.grad, rdq, dtype, "bwd")
    close(kk.grad, rdk, dtype, "bwd")
    close(vv.grad, rdv, dtype, "bwd")
