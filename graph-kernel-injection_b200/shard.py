"""(batch, head) sharding across ranks, backend-agnostic.

Every (batch, head) pair of the attention is independent (the block mask is
shared by all heads, upstream sparse_triton_kernel.py:645-650), so ranks split
the flattened b*H + h index range contiguously and need no collective on the
data path.  The helpers below are what a multi-GPU driver needs around that:
the split, a max-over-ranks reduction for timing, and a gather of small
verification values.  They take an optional process group and work with any
backend (NCCL on GPUs, gloo on CPU).
"""

from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


def shard_units(total: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, stop) of `total` units for `rank` of `world`;
    the first `total % world` ranks take one extra unit."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    if total < 0:
        raise ValueError("total must be non-negative")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def bh_slice(x: torch.Tensor, start: int, stop: int) -> torch.Tensor:
    """Rows [start, stop) of the flattened (batch, head) axes of a
    [B, H, N, D] tensor, as a [1, stop - start, N, D] view."""
    B, H = x.shape[:2]
    return x.reshape(B * H, *x.shape[2:])[start:stop].unsqueeze(0)


def _device_for(group) -> torch.device:
    backend = dist.get_backend(group)
    return torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" \
        else torch.device("cpu")


def max_over_ranks(value: float, group: Optional[dist.ProcessGroup] = None) -> float:
    """Largest `value` over all ranks (the job time of a timed region)."""
    if not dist.is_initialized():
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=_device_for(group))
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def gather_values(values: Sequence[float],
                  group: Optional[dist.ProcessGroup] = None) -> List[List[float]]:
    """Every rank's `values` (same length on all ranks), in rank order."""
    if not dist.is_initialized():
        return [list(map(float, values))]
    t = torch.tensor(list(values), dtype=torch.float64, device=_device_for(group))
    out = [torch.empty_like(t) for _ in range(dist.get_world_size(group))]
    dist.all_gather(out, t, group=group)
    return [o.tolist() for o in out]
