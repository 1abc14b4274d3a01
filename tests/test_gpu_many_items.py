"""Problems with several work items per SM.

``dq_gemm_kernel`` is persistent: one CTA per SM walks the (query tile,
query (b, h)) items, streaming (dS, K) pairs through one ring across item
boundaries, alternating two TMEM accumulators and storing an item's dQ while
the next accumulates.  The small parity cases give every CTA one item; here
B * H * query tiles is several times the SM count, with query tiles that see
no key scattered between the others (items that take no accumulator), so
every CTA crosses item boundaries, reuses both accumulators and its staging
tile, and skips empty items.  Each head's O and dQ must equal, bit for bit,
the same head run alone (one item per CTA); two heads are also checked
against the float64 oracle, gradients included.  At head_dim 64 the backward
recomputes dQ (``dq_tc_kernel``) instead of storing dS, so that case checks
the same properties on the non-persistent kernels.
"""

from __future__ import annotations

import pytest
import torch

import sbfa_native as native
import sparse_triton_kernel as stk
from oracle import streaming_oracle as orc
from tests.parity import check_half

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _step(q, k, v, do, mask, kw):
    q, k, v = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    o = stk.block_sparse_attention(q, k, v, mask, **kw)
    o.backward(do)
    return o.detach(), q.grad, k.grad, v.grad


@pytest.mark.parametrize("D", [128, 64])
def test_items_beyond_sm_count_match_single_heads(D):
    B, H, N, bm, S, W = 1, 16, 4096, 128, 4, 256
    dt = torch.bfloat16
    items = B * H * (N // bm)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert items >= 3 * sms, "the case must give every CTA three or more items"
    g = torch.Generator(device=DEV).manual_seed(21)
    q, k, v, do = (torch.randn(B, H, N, D, generator=g, device=DEV, dtype=dt) for _ in range(4))
    mask = stk.make_streaming_mask(N, N, stk.StreamingMaskSpec(S, W), bm, bm, DEV).clone()
    mask[5::7, :] = 0  # query tiles with no kept block between the others
    kw = dict(block_m=bm, block_n=bm, is_causal=True, sink_size=S, window_size=W)

    o, dq, dk, dv = _step(q, k, v, do, mask, kw)
    torch.cuda.synchronize()
    assert native.device_status() == 0
    for h in range(H):
        sl = slice(h, h + 1)
        o1, dq1, dk1, dv1 = _step(q[:, sl].contiguous(), k[:, sl].contiguous(),
                                  v[:, sl].contiguous(), do[:, sl].contiguous(), mask, kw)
        assert torch.equal(o[:, sl], o1), f"O of head {h} differs from the head run alone"
        assert torch.equal(dq[:, sl], dq1), f"dQ of head {h} differs from the head run alone"
        for nm, a, b in (("dK", dk[:, sl], dk1), ("dV", dv[:, sl], dv1)):
            check_half(a, b.double(), dt, f"{nm} head {h} vs alone")
    for h in (0, H - 1):
        sl = slice(h, h + 1)
        ref = orc.attention_forward_backward(
            *(t[:, sl].double().cpu() for t in (q, k, v, do)), mask.cpu(), **kw)
        for nm, a, b in zip(("O", "dQ", "dK", "dV"), (o, dq, dk, dv), ref):
            check_half(a[:, sl], b, dt, f"{nm} head {h} vs oracle")
        zero_rows = torch.zeros(N, dtype=torch.bool)
        for ti in range(5, N // bm, 7):
            zero_rows[ti * bm:(ti + 1) * bm] = True
        assert torch.equal(dq[:, sl, zero_rows.to(DEV)], torch.zeros_like(dq[:, sl, zero_rows.to(DEV)]))
    assert native.device_status() == 0
