"""Multi-rank host logic on CPU with gloo (world size 2).

(batch, head) sharding: each rank computes its contiguous slice of the
heads (here with the CPU oracle standing in for the device kernels) and the
gathered slices equal the single-process result; max-over-ranks timing; and
a rank that fails before a collective makes the other rank's collective end
with an error instead of hanging.
"""

from __future__ import annotations

import datetime
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "graph-kernel-injection_b200")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    for p in (ROOT, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _shard_worker(rank, world, port, q):
    _init(rank, world, port)
    import shard
    from oracle import streaming_oracle as orc
    B, H, N, D = 2, 3, 96, 16
    g = torch.Generator().manual_seed(0)
    qq, kk, vv = (torch.randn(B, H, N, D, generator=g, dtype=torch.float64) for _ in range(3))
    mask = orc.make_streaming_mask(N, N, 4, 24, 32, 32)
    start, stop = shard.shard_units(B * H, world, rank)
    out = orc.attention_forward(shard.bh_slice(qq, start, stop), shard.bh_slice(kk, start, stop),
                                shard.bh_slice(vv, start, stop), mask, block_m=32, block_n=32,
                                is_causal=True, sink_size=4, window_size=24)
    # gather variable-size slices: pad to the largest shard
    size = torch.tensor([stop - start])
    sizes = [torch.zeros_like(size) for _ in range(world)]
    dist.all_gather(sizes, size)
    cap = int(max(s.item() for s in sizes))
    padded = torch.zeros(cap, N, D, dtype=torch.float64)
    padded[: stop - start] = out[0]
    parts = [torch.zeros_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded)
    t_max = shard.max_over_ranks(float(rank + 1))
    vals = shard.gather_values([float(rank), float(out.sum())])
    if rank == 0:
        full = orc.attention_forward(qq, kk, vv, mask, block_m=32, block_n=32, is_causal=True,
                                     sink_size=4, window_size=24).reshape(B * H, N, D)
        got = torch.cat([p[: int(s.item())] for p, s in zip(parts, sizes)])
        q.put((torch.allclose(got, full, atol=1e-12), t_max, vals))
    dist.destroy_process_group()


def _failing_worker(rank, world, port, q):
    _init(rank, world, port, timeout_s=5)
    try:
        if rank == 1:
            raise RuntimeError("rank 1 fails before the collective")
        t = torch.ones(4)
        dist.all_reduce(t)
        q.put(("no error", None))
    except RuntimeError as e:
        q.put((type(e).__name__, str(e)[:200]))
    finally:
        if rank == 1:
            q.close()
            q.join_thread()  # flush the result before leaving
            os._exit(0)      # leave without joining the collective


def test_shard_units_cover_everything():
    sys.path.insert(0, PKG)
    import shard
    for total in (0, 1, 7, 128, 2048):
        for world in (1, 2, 3, 8):
            ranges = [shard.shard_units(total, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard.shard_units(4, 2, 2)


def test_two_gloo_ranks_reassemble_the_full_result():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    ok, t_max, vals = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert ok
    assert t_max == 2.0
    assert [v[0] for v in vals] == [0.0, 1.0]


def test_failed_rank_ends_the_collective_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    kinds = sorted(r[0] for r in results)
    assert "no error" not in kinds, results
