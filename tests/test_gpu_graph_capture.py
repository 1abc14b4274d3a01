"""The forward + backward step captured in a CUDA graph.

``block_sparse_attention`` launches only libsbfa kernels on torch's current
stream, allocates its outputs and workspaces through torch, and reads the
host copy of a plan's tile count only when the plan is built (cached per
mask), so after one eager call the whole training step (forward, Delta,
dK/dV, dQ) can be captured with ``torch.cuda.graph`` and replayed; the
bench times its headline that way.  Replays must give the same bits as the
eager step on the same inputs, and must follow new values written into the
captured input tensors.
"""

from __future__ import annotations

import pytest
import torch

import sparse_triton_kernel as stk
from oracle import streaming_oracle as orc
from tests.parity import check_half

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.mark.parametrize("D,bm,kv_heads", [(128, 128, 4), (64, 64, 4), (128, 128, 2)])
def test_fwd_bwd_graph_replay_matches_eager(D, bm, kv_heads):
    B, H, N, S, W = 1, 4, 1000, 4, 256
    dt = torch.bfloat16
    g = torch.Generator(device=DEV).manual_seed(11)
    q = torch.randn(B, H, N, D, generator=g, device=DEV, dtype=dt).requires_grad_(True)
    k = torch.randn(B, kv_heads, N, D, generator=g, device=DEV, dtype=dt).requires_grad_(True)
    v = torch.randn(B, kv_heads, N, D, generator=g, device=DEV, dtype=dt).requires_grad_(True)
    do = torch.randn(B, H, N, D, generator=g, device=DEV, dtype=dt)
    mask = stk.make_streaming_mask(N, N, stk.StreamingMaskSpec(S, W), bm, bm, DEV)
    kw = dict(block_m=bm, block_n=bm, is_causal=True, sink_size=S, window_size=W)

    def step():
        for t in (q, k, v):
            t.grad = None
        o = stk.block_sparse_attention(q, k, v, mask, **kw)
        o.backward(do)
        return o

    # eager reference (this call also builds and caches the plans)
    o_e = step().detach().clone()
    grads_e = [t.grad.detach().clone() for t in (q, k, v)]

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode="thread_local"):
        o_g = step()
    grads_g = [q.grad, k.grad, v.grad]

    for _ in range(2):  # two replays in a row: no state carried between them
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(o_g, o_e), "O differs between graph replay and eager step"
        for nm, a, b in zip(("dQ", "dK", "dV"), grads_g, grads_e):
            assert torch.equal(a, b), f"{nm} differs between graph replay and eager step"

    # new inputs written in place are picked up by the next replay
    with torch.no_grad():
        q.mul_(0.5)
        v.add_(0.25)
    graph.replay()
    torch.cuda.synchronize()
    rep = H // kv_heads  # query head h reads key/value head h // rep
    ref = orc.attention_forward(q.detach().double().cpu(),
                                k.detach().double().cpu().repeat_interleave(rep, dim=1),
                                v.detach().double().cpu().repeat_interleave(rep, dim=1),
                                mask.cpu(), None, bm, bm, True, S, W)
    check_half(o_g.detach(), ref, dt, "O after in-place input update")
    del graph
