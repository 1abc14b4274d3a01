"""Failure detection without a GPU fault: a bounded wait that nothing ever
satisfies gives up after its limit, the status word reports it to the host,
and the context keeps working (the next attention call is correct and clean).
Same wait primitive as every pipeline barrier of the tensor-core kernels."""

from __future__ import annotations

import time

import pytest
import torch

import sbfa_native as native
import sparse_triton_kernel as stk
from oracle import streaming_oracle as orc

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_and_context_survives():
    lib = native.lib()
    assert native.device_status() == 0
    t0 = time.perf_counter()
    native.check(lib.sbfa_selftest_wait_timeout(20_000_000, native.stream_ptr("cuda")),
                 "selftest")
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert 0.015 < elapsed < 5.0
    assert native.device_status() == 1   # kStatusWaitTimeout, read and cleared
    assert native.device_status() == 0
    # the context is intact: an ordinary call still matches the oracle
    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v = (torch.randn(1, 2, 256, 128, generator=g, device="cuda", dtype=torch.bfloat16)
               for _ in range(3))
    mask = stk.make_streaming_mask(256, 256, stk.StreamingMaskSpec(4, 64), 128, 128, "cuda")
    o = stk.block_sparse_attention(q, k, v, mask, block_m=128, block_n=128, is_causal=True,
                                   sink_size=4, window_size=64)
    ref = orc.attention_forward(q.double().cpu(), k.double().cpu(), v.double().cpu(), mask.cpu(),
                                block_m=128, block_n=128, is_causal=True, sink_size=4,
                                window_size=64)
    assert (o.double().cpu() - ref).abs().max().item() < 2e-2
    assert native.device_status() == 0


def test_selftest_rejects_bad_limit():
    assert native.lib().sbfa_selftest_wait_timeout(5, None) == 1
