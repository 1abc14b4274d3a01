"""StreamingLLM sink+window block-sparse attention on B200 (sm_100a).

Drop-in replacement for the upstream module of the same name
(Hridambiswas/graph-kernel-injection ``sparse_triton_kernel.py``).  The
module name is kept so every ``from sparse_triton_kernel import ...``
call site -- including ``fx_compiler_pass`` -- works unchanged.  There is
no Triton here: forward, backward and decode run hand-written CUDA in
``libsbfa.so`` (see ``include/sbfa.h``), reached through ctypes
(``sbfa_native``).  If the library is missing the attention entry points
raise ``RuntimeError``; there is no CPU fallback.

Public API (same names, arguments and error behaviour as upstream):

* :class:`StreamingMaskSpec`            upstream ``:81-101``
* :func:`make_streaming_mask`           upstream ``:104-181``
* :func:`make_dense_mask`               upstream ``:184-210``
* :func:`block_sparse_attention`        upstream ``:787-837``
* :class:`_BlockSparseFlashAttention`   upstream ``:609-779``
* :func:`reference_block_sparse_attention` upstream ``:845-902`` (eager
  Θ(N²) function kept for API compatibility; never used by the kernels)
* :func:`streaming_token_mask`          upstream ``:905-932``

Semantics: queries are bottom-right aligned (query row ``r`` is absolute
position ``n_kv - n_q + r``); a kept block applies the token rule
``(k <= q) & (k < S | k >= q - W + 1)`` when ``is_causal``; rows with no
visible key give ``O = 0`` and zero gradients.
"""

from __future__ import annotations

import ctypes
import math
import os
import weakref
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch

import sbfa_native as native

# ---------------------------------------------------------------------------
# Mask construction
# ---------------------------------------------------------------------------


@dataclass(frozen=True)
class StreamingMaskSpec:
    """StreamingLLM sparsity parameters: ``sink_size`` leading tokens every
    query sees, and a causal window of ``window_size`` recent tokens
    (a query at ``q`` sees keys ``[q - W + 1, q]``)."""

    sink_size: int
    window_size: int

    def __post_init__(self) -> None:
        if self.sink_size < 0 or self.window_size < 0:
            raise ValueError("sink_size and window_size must be non-negative")


def _is_cuda(device) -> bool:
    return torch.device(device).type == "cuda"


def make_streaming_mask(n_q: int, n_kv: int, spec: StreamingMaskSpec, block_m: int,
                        block_n: int, device: torch.device | str = "cuda") -> torch.Tensor:
    """Block-level StreamingLLM mask, int32 ``[ceil(n_q/BM), ceil(n_kv/BN)]``.

    Entry ``(i, j)`` is 1 iff ``q_hi > k_lo`` and (``k_lo < S`` or
    ``k_hi - 1 >= q_lo - W + 1``) with ``q_lo = i*BM + n_kv - n_q``,
    ``q_hi = q_lo + BM``, ``k_lo = j*BN``, ``k_hi = k_lo + BN`` (unclamped).
    On a CUDA device the mask is built by the ``sbfa_streaming_mask`` kernel;
    a host tensor is computed on the host.
    """
    if n_q <= 0 or n_kv <= 0:
        raise ValueError("n_q and n_kv must be positive")
    n_qb = (n_q + block_m - 1) // block_m
    n_kb = (n_kv + block_n - 1) // block_n
    if _is_cuda(device):
        dev = torch.device(device)
        out = torch.empty((n_qb, n_kb), dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            native.check(native.lib().sbfa_streaming_mask(
                n_q, n_kv, spec.sink_size, spec.window_size, block_m, block_n,
                out.data_ptr(), native.stream_ptr(dev)), "streaming_mask")
        return out
    i = torch.arange(n_qb, dtype=torch.int64, device=device)
    j = torch.arange(n_kb, dtype=torch.int64, device=device)
    first_q = i * block_m + (n_kv - n_q)           # q_lo
    last_k = j * block_n + (block_n - 1)            # k_hi - 1
    keep = ((first_q[:, None] + block_m) > (j * block_n)[None, :]) & (
        ((j * block_n) < spec.sink_size)[None, :]
        | (last_k[None, :] >= (first_q[:, None] - spec.window_size + 1)))
    return keep.to(torch.int32).contiguous()


def make_dense_mask(n_q: int, n_kv: int, block_m: int, block_n: int, causal: bool = False,
                    device: torch.device | str = "cuda") -> torch.Tensor:
    """Fully dense (or dense-causal: ``k_lo < q_hi``) block mask."""
    if n_q % block_m != 0 or n_kv % block_n != 0:
        raise ValueError("block_m / block_n must divide n_q / n_kv")
    n_qb, n_kb = n_q // block_m, n_kv // block_n
    if _is_cuda(device):
        dev = torch.device(device)
        out = torch.empty((n_qb, n_kb), dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            native.check(native.lib().sbfa_dense_mask(
                n_q, n_kv, block_m, block_n, int(bool(causal)), out.data_ptr(),
                native.stream_ptr(dev)), "dense_mask")
        return out
    if not causal:
        return torch.ones((n_qb, n_kb), dtype=torch.int32, device=device)
    rows_end = (torch.arange(n_qb, device=device) + 1) * block_m
    cols_start = torch.arange(n_kb, device=device) * block_n
    return (cols_start[None, :] < rows_end[:, None]).to(torch.int32).contiguous()


def streaming_token_mask(n_q: int, n_kv: int, sink_size: int, window_size: int,
                         device: torch.device | str = "cpu") -> torch.Tensor:
    """Exact token-level StreamingLLM mask, bool ``[n_q, n_kv]``."""
    qpos = torch.arange(n_kv - n_q, n_kv, device=device)[:, None]
    kpos = torch.arange(n_kv, device=device)[None, :]
    return (kpos <= qpos) & ((kpos < sink_size) | (kpos >= qpos - window_size + 1))


# ---------------------------------------------------------------------------
# Plans: compacted kept-tile lists, cached per mask tensor
# ---------------------------------------------------------------------------


class _PlanCache:
    """Per-mask cache of device plans, keyed by the mask object, its
    in-place version counter, the sequence geometry and the tile sizes.
    Entries die with the mask tensor."""

    def __init__(self) -> None:
        self._by_id: Dict[int, Tuple[weakref.ref, Dict[tuple, dict]]] = {}

    def get(self, mask: torch.Tensor, key: tuple, build):
        ent = self._by_id.get(id(mask))
        if ent is None or ent[0]() is not mask:
            mid = id(mask)
            ref = weakref.ref(mask, lambda _r, mid=mid: self._by_id.pop(mid, None))
            ent = (ref, {})
            self._by_id[mid] = ent
        full_key = (mask._version,) + key
        plan = ent[1].get(full_key)
        if plan is None:
            # an in-place write to the mask invalidates plans of older versions
            for stale in [k for k in ent[1] if k[0] != mask._version]:
                del ent[1][stale]
            plan = build()
            ent[1][full_key] = plan
        return plan


_PLANS = _PlanCache()


def build_plan(mask: torch.Tensor, n_q: int, n_kv: int, block_m: int, block_n: int,
               tile_m: int, tile_n: int) -> dict:
    """Run ``sbfa_build_plan`` on a device int32 mask (CSR + CSC lists)."""
    dev = mask.device
    n_ti = (n_q + tile_m - 1) // tile_m
    n_tj = (n_kv + tile_n - 1) // tile_n
    cap = max(1, n_ti * n_tj)
    if cap >= 2 ** 31:
        raise ValueError("tile grid too large for int32 plan indices")
    i32 = dict(dtype=torch.int32, device=dev)
    plan = {
        "row_ptr": torch.empty(n_ti + 1, **i32), "col_idx": torch.empty(cap, **i32),
        "col_ptr": torch.empty(n_tj + 1, **i32), "row_idx": torch.empty(cap, **i32),
        "nnz": torch.empty(1, **i32), "tiles": (tile_m, tile_n),
    }
    with torch.cuda.device(dev):
        native.check(native.lib().sbfa_build_plan(
            mask.data_ptr(), n_q, n_kv, block_m, block_n, tile_m, tile_n,
            plan["row_ptr"].data_ptr(), plan["col_idx"].data_ptr(),
            plan["col_ptr"].data_ptr(), plan["row_idx"].data_ptr(), plan["nnz"].data_ptr(),
            native.stream_ptr(dev)), "build_plan")
    return plan


def _plan_for(mask: torch.Tensor, pass_id: int, dtype: torch.dtype, head_dim: int, n_q: int,
              n_kv: int, block_m: int, block_n: int) -> dict:
    tm, tn = native.plan_tiles(pass_id, dtype, head_dim, n_q)
    key = (n_q, n_kv, block_m, block_n, tm, tn)
    return _PLANS.get(mask, key, lambda: build_plan(mask, n_q, n_kv, block_m, block_n, tm, tn))


def _plan_nnz(plan: dict) -> int:
    """Kept tiles of a plan on the host (read once per plan)."""
    if "nnz_host" not in plan:
        plan["nnz_host"] = int(plan["nnz"].item())
    return plan["nnz_host"]


def _csc_positions(plan: dict, dev: torch.device) -> torch.Tensor:
    """For every CSR entry of a plan, the CSC position of the same tile
    (built once per plan): where the dK/dV pass stores that tile's dS."""
    if "csc_pos" not in plan:
        pos = torch.empty_like(plan["col_idx"])
        native.check(native.lib().sbfa_plan_csc_positions(
            plan["row_ptr"].data_ptr(), plan["col_idx"].data_ptr(), plan["col_ptr"].data_ptr(),
            plan["row_idx"].data_ptr(), plan["row_ptr"].numel() - 1, pos.data_ptr(),
            native.stream_ptr(dev)), "plan_csc_positions")
        plan["csc_pos"] = pos
    return plan["csc_pos"]


DS_BUDGET_ENV = "SBFA_BWD_DS_MAX_BYTES"


def _ds_budget(dev: torch.device) -> int:
    """Most device bytes a backward call may take for stored dS tiles:
    ``SBFA_BWD_DS_MAX_BYTES`` when set (0 keeps the recomputing dQ kernel),
    else a quarter of the device's memory, at most half of what is free."""
    env = os.environ.get(DS_BUDGET_ENV)
    if env is not None:
        return int(env)
    free, total = torch.cuda.mem_get_info(dev)
    return min(total // 4, free // 2)


# ---------------------------------------------------------------------------
# Autograd bridge
# ---------------------------------------------------------------------------


def _validate(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_mask: torch.Tensor,
              block_m: int, block_n: int) -> Tuple[int, int, int, int, int]:
    """Input checks of upstream ``sparse_triton_kernel.py:631-649``."""
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("Q/K/V must be 4-D [B, H, N, D] tensors")
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise ValueError("All inputs must live on a CUDA device")
    B, H, N_Q, D = q.shape
    N_KV = k.shape[2]
    if k.shape != v.shape:
        raise ValueError("K and V must share shape")
    # grouped-query attention (an extension: upstream requires equal head
    # counts): K/V may have fewer heads than Q when they divide Q's count
    if k.shape[0] != B or k.shape[-1] != D or H % k.shape[1] != 0:
        raise ValueError("Q/K/V batch/head/dim mismatch")
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError("Q/K/V must share dtype")
    if not (q.device == k.device == v.device):
        raise ValueError("Q/K/V must live on the same device")
    if block_m <= 0 or block_n <= 0:
        raise ValueError("block_m and block_n must be positive")
    n_qb = (N_Q + block_m - 1) // block_m
    n_kb = (N_KV + block_n - 1) // block_n
    if tuple(block_mask.shape) != (n_qb, n_kb):
        raise ValueError(f"block_mask has shape {tuple(block_mask.shape)}, "
                         f"expected {(n_qb, n_kb)}")
    return B, H, N_Q, N_KV, D


_TC_DTYPES = (torch.float16, torch.bfloat16)


def _strides3(t: torch.Tensor) -> List[int]:
    """(batch, head, row) element strides of a [B, H, N, D] tensor whose last
    dimension is unit-stride; a size-1 dimension gets the extent of the
    dimensions inside it (any stride is valid there, and this one also
    satisfies the tensor-core alignment rules whenever the others do)."""
    shape, st = t.shape, list(t.stride())
    out = []
    for i in range(3):
        if shape[i] == 1:
            out.append(max(st[j] * shape[j] for j in range(i + 1, 4)))
        else:
            out.append(st[i])
    return out


def _readable(t: torch.Tensor, tensor_core: bool) -> torch.Tensor:
    """``t`` itself when the kernels can read it in place, else a contiguous
    copy (upstream always copies: ``sparse_triton_kernel.py:707, 834``).
    Reads may overlap (an expanded dimension is fine for the CUDA-core
    kernels); the tensor-core kernels read through TMA, which needs a 16-byte
    aligned base and strides that are positive multiples of 8 elements."""
    if t.stride(-1) != 1 and t.shape[-1] != 1:
        return t.contiguous()
    if t.is_contiguous():
        return t
    st = _strides3(t)
    if st[2] < t.shape[-1] or min(st) < 0:
        return t.contiguous()
    if tensor_core and (t.data_ptr() % 16 or any(x <= 0 or x % 8 for x in st)):
        return t.contiguous()
    return t


def _uses_tensor_cores(dtype: torch.dtype, d: int) -> bool:
    return dtype in _TC_DTYPES and d in (64, 128)


def _stride_array(*ts: torch.Tensor):
    vals = [x for t in ts for x in _strides3(t)]
    return (ctypes.c_int64 * len(vals))(*vals)


class _BlockSparseFlashAttention(torch.autograd.Function):
    """Autograd bridge to the libsbfa forward / decode / backward kernels
    (upstream ``sparse_triton_kernel.py:609-779``)."""

    @staticmethod
    def forward(ctx, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                block_mask: torch.Tensor, softmax_scale: float, block_m: int, block_n: int,
                is_causal: bool, sink_size: int, window_size: int) -> torch.Tensor:
        native.lib()  # raises RuntimeError when the CUDA library is absent
        B, H, N_Q, N_KV, D = _validate(q, k, v, block_mask, block_m, block_n)
        native.dtype_code(q.dtype)
        dev = q.device
        block_mask = block_mask.to(device=dev, dtype=torch.int32).contiguous()
        code = native.dtype_code(q.dtype)
        L = native.lib()
        kv_heads = int(k.shape[1])
        decode = N_Q == 1 and bool(L.sbfa_decode_supported(code, D))
        if decode:  # the decode kernel reads contiguous q / k / v
            q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        else:       # strided views are read in place
            tcore = _uses_tensor_cores(q.dtype, D)
            q, k, v = (_readable(t, tcore) for t in (q, k, v))
        o = torch.empty((B, H, N_Q, D), dtype=q.dtype, device=dev)
        lse = torch.empty((B, H, N_Q), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            stream = native.stream_ptr(dev)
            if decode:
                plan = _plan_for(block_mask, 3, q.dtype, D, N_Q, N_KV, block_m, block_n)
                ws_bytes = int(L.sbfa_decode_workspace_bytes(B, H, N_KV, D, block_n))
                ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
                native.check(L.sbfa_decode(
                    q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                    B, H, N_KV, D, code, float(softmax_scale), int(bool(is_causal)),
                    int(sink_size), int(window_size), block_mask.data_ptr(), block_m, block_n,
                    plan["row_ptr"].data_ptr(), plan["col_idx"].data_ptr(), ws.data_ptr(),
                    ws.numel(), kv_heads, stream), "decode")
            else:
                plan = _plan_for(block_mask, 0, q.dtype, D, N_Q, N_KV, block_m, block_n)
                native.check(L.sbfa_fwd(
                    q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                    B, H, N_Q, N_KV, D, code, float(softmax_scale), int(bool(is_causal)),
                    int(sink_size), int(window_size), block_mask.data_ptr(), block_m, block_n,
                    plan["row_ptr"].data_ptr(), plan["col_idx"].data_ptr(),
                    _stride_array(q, k, v, o), kv_heads, stream), "fwd")
        ctx.save_for_backward(q, k, v, o, lse, block_mask)
        ctx.softmax_scale = float(softmax_scale)
        ctx.block_m = int(block_m)
        ctx.block_n = int(block_n)
        ctx.is_causal = bool(is_causal)
        ctx.sink_size = int(sink_size)
        ctx.window_size = int(window_size)
        ctx.q_offset = int(N_KV - N_Q)
        return o

    @staticmethod
    def backward(ctx, do: torch.Tensor) -> Tuple[Optional[torch.Tensor], ...]:
        q, k, v, o, lse, block_mask = ctx.saved_tensors
        if do.dtype != q.dtype:
            do = do.to(q.dtype)
        B, H, N_Q, D = q.shape
        N_KV = k.shape[2]
        dev = q.device
        tcore = _uses_tensor_cores(q.dtype, D)
        do = _readable(do, tcore)
        # gradients in the layout of their inputs, so they flow back through
        # the caller's transposes without a copy
        dq, dk, dv = (_readable(torch.empty_like(t), tcore) for t in (q, k, v))
        delta = torch.empty((B, H, N_Q), dtype=torch.float32, device=dev)
        L = native.lib()
        kv_heads = int(k.shape[1])
        code = native.dtype_code(q.dtype)
        ws_bytes = int(L.sbfa_bwd_workspace_bytes(B, H, D, code, kv_heads))
        split_ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
        with torch.cuda.device(dev):
            p_dq = _plan_for(block_mask, 1, q.dtype, D, N_Q, N_KV, ctx.block_m, ctx.block_n)
            p_kv = _plan_for(block_mask, 2, q.dtype, D, N_Q, N_KV, ctx.block_m, ctx.block_n)
            # the dK/dV pass stores dS for a dQ GEMM when the tiles fit the budget
            ds_ws, ds_bytes, csc = None, 0, None
            if p_dq is p_kv:
                need = int(L.sbfa_bwd_ds_workspace_bytes(B, H, D, code, _plan_nnz(p_dq)))
                if 0 < need <= _ds_budget(dev):
                    ds_ws = torch.empty(need, dtype=torch.uint8, device=dev)
                    csc, ds_bytes = _csc_positions(p_dq, dev), need
            native.check(L.sbfa_bwd(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                do.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), delta.data_ptr(),
                B, H, N_Q, N_KV, D, code, ctx.softmax_scale,
                int(ctx.is_causal), ctx.sink_size, ctx.window_size, block_mask.data_ptr(),
                ctx.block_m, ctx.block_n, p_dq["row_ptr"].data_ptr(),
                p_dq["col_idx"].data_ptr(), p_kv["col_ptr"].data_ptr(),
                p_kv["row_idx"].data_ptr(), _stride_array(q, k, v, o, do, dq, dk, dv),
                kv_heads, native.ptr(split_ws), ws_bytes, native.ptr(csc),
                _plan_nnz(p_dq) if csc is not None else 0, native.ptr(ds_ws), ds_bytes,
                native.stream_ptr(dev)), "bwd")
        return dq, dk, dv, None, None, None, None, None, None, None


def block_sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           block_mask: torch.Tensor, softmax_scale: Optional[float] = None,
                           block_m: int = 64, block_n: int = 64, is_causal: bool = False,
                           sink_size: int = 0, window_size: int = 0) -> torch.Tensor:
    """Differentiable block-sparse attention over ``[B, H, N, D]`` CUDA tensors.

    ``block_mask`` is ``[ceil(N_Q/block_m), ceil(N_KV/block_n)]`` (coerced
    to int32); a nonzero entry keeps the block.  With ``is_causal`` every
    kept block also applies the StreamingLLM token rule with
    ``sink_size`` / ``window_size``.  ``softmax_scale`` defaults to
    ``1/sqrt(D)``.  A single query (``N_Q == 1``) runs the split-KV decode
    kernel, which with grouped K/V heads reads each K/V row once for all the
    query heads of its group.
    """
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(q.shape[-1])
    return _BlockSparseFlashAttention.apply(
        q, k, v, block_mask, float(softmax_scale), int(block_m), int(block_n), bool(is_causal),
        int(sink_size), int(window_size))


# ---------------------------------------------------------------------------
# Eager function (API compatibility)
# ---------------------------------------------------------------------------


def reference_block_sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                     block_mask: torch.Tensor,
                                     softmax_scale: Optional[float] = None, block_m: int = 64,
                                     block_n: int = 64, is_causal: bool = False,
                                     sink_size: int = 0, window_size: int = 0) -> torch.Tensor:
    """Eager Θ(N²) masked attention with the same semantics as
    :func:`block_sparse_attention` (upstream ``:845-902``).

    Kept so code written against the upstream module finds it; it is a
    plain torch computation on whatever device its inputs live on and is
    never called by :func:`block_sparse_attention`.
    """
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(q.shape[-1])
    n_q, n_kv = q.shape[-2], k.shape[-2]
    keep = block_mask.to(device=q.device, dtype=torch.bool)
    keep = keep.repeat_interleave(block_m, dim=0).repeat_interleave(block_n, dim=1)
    keep = keep[:n_q, :n_kv]
    if is_causal:
        keep = keep & streaming_token_mask(n_q, n_kv, sink_size, window_size, device=q.device)
    logits = (q @ k.transpose(-2, -1)) * softmax_scale
    probs = torch.softmax(logits.masked_fill(~keep, float("-inf")), dim=-1)
    return torch.nan_to_num(probs, nan=0.0) @ v


__all__ = [
    "StreamingMaskSpec",
    "block_sparse_attention",
    "make_dense_mask",
    "make_streaming_mask",
    "reference_block_sparse_attention",
    "streaming_token_mask",
]
