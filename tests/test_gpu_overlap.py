"""The backward with the dQ GEMM overlapped on a side stream.

At head_dim 128 the backward cuts the (b, h) units into groups and runs
group g's dQ GEMM on a high-priority side stream beside group g + 1's dK/dV
pass (automatic once the problem has 64 query-tile items per SM;
``SBFA_BWD_GROUPS`` forces a group count, 1 switching the overlap off).
Every group computes exactly what the single pass computes for its units,
so the results must be bit-identical with and without the overlap, for
whole-batch groups, for head-range groups, under grouped-query attention,
and inside a captured CUDA graph (the capture takes the side stream in and
joins it again).
"""

from __future__ import annotations

import os

import pytest
import torch

import sbfa_native as native
import sparse_triton_kernel as stk
from oracle import streaming_oracle as orc
from tests.parity import check_half

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture
def groups_env():
    old = os.environ.get("SBFA_BWD_GROUPS")
    yield
    if old is None:
        os.environ.pop("SBFA_BWD_GROUPS", None)
    else:
        os.environ["SBFA_BWD_GROUPS"] = old


def _inputs(B, H, kv_heads, N, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    dt = torch.bfloat16
    q = torch.randn(B, H, N, 128, generator=g, device=DEV, dtype=dt)
    k = torch.randn(B, kv_heads, N, 128, generator=g, device=DEV, dtype=dt)
    v = torch.randn(B, kv_heads, N, 128, generator=g, device=DEV, dtype=dt)
    do = torch.randn(B, H, N, 128, generator=g, device=DEV, dtype=dt)
    return q, k, v, do


def _step(q, k, v, do, mask, kw):
    q, k, v = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    o = stk.block_sparse_attention(q, k, v, mask, **kw)
    o.backward(do)
    torch.cuda.synchronize()
    return [o.detach(), q.grad, k.grad, v.grad]


@pytest.mark.parametrize("B,H,kv_heads,groups", [
    (4, 4, 4, 4),    # one batch element per group
    (2, 8, 8, 4),    # two head ranges per batch element
    (1, 8, 2, 8),    # grouped-query attention, ranges of whole K/V groups
    (2, 8, 8, 3),    # a count that does not divide: rounded to what does
])
def test_overlapped_backward_bitwise(groups_env, B, H, kv_heads, groups):
    N, S, W = 2048, 4, 512
    q, k, v, do = _inputs(B, H, kv_heads, N, seed=31)
    mask = stk.make_streaming_mask(N, N, stk.StreamingMaskSpec(S, W), 128, 128, DEV)
    kw = dict(block_m=128, block_n=128, is_causal=True, sink_size=S, window_size=W)
    os.environ["SBFA_BWD_GROUPS"] = "1"
    ref = _step(q, k, v, do, mask, kw)
    os.environ["SBFA_BWD_GROUPS"] = str(groups)
    got = _step(q, k, v, do, mask, kw)
    for nm, a, b in zip(("O", "dQ", "dK", "dV"), got, ref):
        assert torch.equal(a, b), f"{nm} differs between the overlapped and the single pass"
    assert native.device_status() == 0
    # and one head against the oracle
    rep = H // kv_heads
    r = orc.attention_forward_backward(
        q[:1, :1].double().cpu(), k[:1, :1].double().cpu(), v[:1, :1].double().cpu(),
        do[:1, :1].double().cpu(), mask.cpu(), **kw)
    check_half(got[1][:1, :1], r[1], torch.bfloat16, "dQ head 0 vs oracle")
    if rep == 1:
        check_half(got[2][:1, :1], r[2], torch.bfloat16, "dK head 0 vs oracle")


@pytest.mark.parametrize("mode", ["thread_local", "global"])
def test_overlapped_backward_in_cuda_graph(groups_env, mode):
    """The capture runs on a stream no backward call has used before, so
    the backward creates that stream's side stream inside the capture."""
    B, H, N, S, W = 2, 8, 2048, 4, 512
    os.environ["SBFA_BWD_GROUPS"] = "4"
    q0, k0, v0, do = _inputs(B, H, H, N, seed=5)
    q, k, v = (t.clone().requires_grad_(True) for t in (q0, k0, v0))
    mask = stk.make_streaming_mask(N, N, stk.StreamingMaskSpec(S, W), 128, 128, DEV)
    kw = dict(block_m=128, block_n=128, is_causal=True, sink_size=S, window_size=W)

    def step():
        for t in (q, k, v):
            t.grad = None
        o = stk.block_sparse_attention(q, k, v, mask, **kw)
        o.backward(do)
        return o

    o_e = step().detach().clone()
    grads_e = [t.grad.detach().clone() for t in (q, k, v)]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=torch.cuda.Stream(), capture_error_mode=mode):
        o_g = step()
    for _ in range(2):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(o_g, o_e)
        for nm, a, b in zip(("dQ", "dK", "dV"), (q.grad, k.grad, v.grad), grads_e):
            assert torch.equal(a, b), f"{nm} differs between graph replay and eager step"
    del graph
    assert native.device_status() == 0
