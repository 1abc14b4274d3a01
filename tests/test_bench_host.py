"""Host-side pieces of bench.py, on CPU.

bench.py runs only on a GPU box, so these tests import it here (no CUDA
call happens at import time) and check the arithmetic its JSON line rests
on: the kept-block work of config 2 and the per-step roofline accounting
when a kernel launches several times per step (the backward launches dK/dV
and the dQ GEMM once per group of (b, h) units when it overlaps them).
"""

from __future__ import annotations

import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test",
                                                  os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_cfg2_work(bench):
    import sparse_triton_kernel as stk
    c = bench.CFG2
    m = stk.make_streaming_mask(c["N"], c["N"], stk.StreamingMaskSpec(c["S"], c["W"]), c["BM"],
                                c["BN"], device="cpu")
    nnz = int(m.sum())
    assert nnz == 2151
    f = bench.f_fwd(bench.CFG2, nnz)
    assert f == pytest.approx(2.3096e12, rel=1e-4)
    assert 3.5 * f == pytest.approx(8.0837e12, rel=1e-4)


def test_roofline_is_per_step_whatever_the_launch_count(bench):
    pk = {"hbm_gbs": 6554.6, "bf16_tflops": 1637.9, "bf16_tflops_sustained": 1368.9}
    F = 2.3096e12
    steps = 10
    # one dK/dV launch of 4.5 ms per step, or four of 1.125 ms: the same work
    one = {"dkdv_tc_kernel": (45.0, 10), "dq_gemm_kernel": (15.8, 10)}
    four = {"dkdv_tc_kernel": (45.0, 40), "dq_gemm_kernel": (15.8, 40)}
    r1 = bench.roofline(one, F, pk, "measured", steps, workload="cfg2")
    r4 = bench.roofline(four, F, pk, "measured", steps, workload="cfg2")
    assert r1["kernel"] == r4["kernel"] == "dkdv_tc_kernel"
    assert r1["achieved"] == r4["achieved"] == pytest.approx(2 * F / 4.5e-3 / 1e12, rel=1e-3)
    assert r1["frac"] == r4["frac"] < 1.0
    assert r4["launches"] == 40 and r4["ms_per_step"] == pytest.approx(4.5)
    assert r4["avg_launch_ms"] == pytest.approx(1.125)


def test_roofline_decode_bytes_per_step(bench):
    pk = {"hbm_gbs": 6554.6, "bf16_tflops": 1637.9, "bf16_tflops_sustained": 1368.9}
    per = {"decode_split_kernel": (3.45, 10), "decode_merge_kernel": (0.06, 10)}
    r = bench.roofline(per, 0.0, pk, "measured", 10, kv_bytes=2.1517e9, workload="cfg4")
    assert r["bound"] == "hbm"
    assert r["achieved"] == pytest.approx(2.1517e9 / 0.345e-3 / 1e9, rel=1e-3)
