"""CPU oracle for StreamingLLM sink+window block-sparse attention.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
file; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
legs of ``bench.py`` use it, and only as the checker (or, for the
reference arm of ``bench.py``, as the timed CPU implementation).

Every function restates one function of the upstream reference
(Hridambiswas/graph-kernel-injection, ``sparse_triton_kernel.py``) in
plain numpy / torch-CPU code:

* :func:`make_streaming_mask`      -> ``sparse_triton_kernel.py:104-181``
* :func:`make_dense_mask`          -> ``sparse_triton_kernel.py:184-210``
* :func:`streaming_token_mask`     -> ``sparse_triton_kernel.py:905-932``
* :func:`effective_token_mask`     -> ``sparse_triton_kernel.py:876-896``
* :func:`attention_forward`        -> ``sparse_triton_kernel.py:845-902``
* :func:`attention_forward_backward` -> the reference's gradient protocol
  (autograd through the eager path, ``benchmark.py:322-355``)
* :func:`tile_plan`                -> no upstream counterpart; it restates,
  as index lists, which (query tile, key tile) pairs the reference
  kernels visit (``sparse_triton_kernel.py:283-285, 448-449, 563-565``).

Parity pin: ``tests/golden/make_golden.py`` runs the upstream reference
itself and stores its outputs under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks this module against them.
"""

from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import numpy as np
import torch


# ---------------------------------------------------------------------------
# Masks (integer work: numpy, bit-exact)
# ---------------------------------------------------------------------------


def make_streaming_mask(n_q: int, n_kv: int, sink: int, window: int,
                        block_m: int, block_n: int) -> np.ndarray:
    """Block-level StreamingLLM mask, ``int32 [ceil(n_q/BM), ceil(n_kv/BN)]``.

    Restates ``sparse_triton_kernel.py:154-181``: queries are bottom-right
    aligned (``q_offset = n_kv - n_q``); block ranges are half-open and
    NOT clamped to the sequence ends; the block rule is
    ``(q_hi > k_lo) & ((k_lo < S) | (k_hi - 1 >= q_lo - W + 1))``.
    """
    if n_q <= 0 or n_kv <= 0:
        raise ValueError("n_q and n_kv must be positive")
    n_qb = -(-n_q // block_m)
    n_kb = -(-n_kv // block_n)
    q_off = n_kv - n_q
    q_lo = np.arange(n_qb, dtype=np.int64) * block_m + q_off
    q_hi = q_lo + block_m
    k_lo = np.arange(n_kb, dtype=np.int64) * block_n
    k_hi = k_lo + block_n
    causal = q_hi[:, None] > k_lo[None, :]
    sink_b = np.broadcast_to(k_lo[None, :] < sink, (n_qb, n_kb))
    win_b = (k_hi[None, :] - 1) >= (q_lo[:, None] - window + 1)
    return np.ascontiguousarray((causal & (sink_b | win_b)).astype(np.int32))


def make_dense_mask(n_q: int, n_kv: int, block_m: int, block_n: int,
                    causal: bool = False) -> np.ndarray:
    """Dense / dense-causal block mask (``sparse_triton_kernel.py:198-210``)."""
    if n_q % block_m != 0 or n_kv % block_n != 0:
        raise ValueError("block_m / block_n must divide n_q / n_kv")
    n_qb, n_kb = n_q // block_m, n_kv // block_n
    if not causal:
        return np.ones((n_qb, n_kb), dtype=np.int32)
    q_hi = (np.arange(n_qb, dtype=np.int64) + 1) * block_m
    k_lo = np.arange(n_kb, dtype=np.int64) * block_n
    return np.ascontiguousarray((k_lo[None, :] < q_hi[:, None]).astype(np.int32))


def streaming_token_mask(n_q: int, n_kv: int, sink: int, window: int) -> np.ndarray:
    """Token rule ``(k <= q) & ((k < S) | (k >= q - W + 1))``, bool [n_q, n_kv].

    Restates ``sparse_triton_kernel.py:927-932`` with
    ``q = (n_kv - n_q) + row``.
    """
    q = np.arange(n_kv - n_q, n_kv, dtype=np.int64)[:, None]
    k = np.arange(n_kv, dtype=np.int64)[None, :]
    return (k <= q) & ((k < sink) | (k >= q - window + 1))


def lift_block_mask(block_mask: np.ndarray, n_q: int, n_kv: int,
                    block_m: int, block_n: int) -> np.ndarray:
    """Block mask lifted to tokens (``sparse_triton_kernel.py:877-879``)."""
    bm = np.asarray(block_mask) != 0
    lifted = np.repeat(np.repeat(bm, block_m, axis=0), block_n, axis=1)
    return lifted[:n_q, :n_kv]


def effective_token_mask(block_mask: np.ndarray, n_q: int, n_kv: int,
                         block_m: int, block_n: int, is_causal: bool,
                         sink: int, window: int) -> np.ndarray:
    """``lifted & token`` when causal, else ``lifted`` (ref ``:876-896``)."""
    lifted = lift_block_mask(block_mask, n_q, n_kv, block_m, block_n)
    if not is_causal:
        return lifted
    return lifted & streaming_token_mask(n_q, n_kv, sink, window)


# ---------------------------------------------------------------------------
# Tile plans: which tile pairs a kernel with (TM, TN) tiles must visit
# ---------------------------------------------------------------------------


def tile_plan(block_mask: np.ndarray, n_q: int, n_kv: int, block_m: int,
              block_n: int, tile_m: int, tile_n: int) -> Dict[str, np.ndarray]:
    """Compacted kept-tile lists for a re-tiling of a user block mask.

    Tile ``(I, J)`` covers query rows ``[I*TM, (I+1)*TM) & [0, n_q)`` and
    key columns ``[J*TN, (J+1)*TN) & [0, n_kv)``.  It is *kept* iff any user
    block it overlaps is nonzero, and *full* iff every user block it
    overlaps is nonzero.  Returns CSR (``row_ptr``, ``col_idx``) and CSC
    (``col_ptr``, ``row_idx``) in ascending index order, with the
    "partial" flag (not full) in bit 31 of each index, exactly the
    encoding the CUDA plan builder emits.
    """
    bm = np.asarray(block_mask) != 0
    n_ti = -(-n_q // tile_m)
    n_tj = -(-n_kv // tile_n)
    kept = np.zeros((n_ti, n_tj), dtype=bool)
    full = np.zeros((n_ti, n_tj), dtype=bool)
    for ti in range(n_ti):
        r0, r1 = ti * tile_m, min((ti + 1) * tile_m, n_q)
        b0, b1 = r0 // block_m, (r1 - 1) // block_m
        for tj in range(n_tj):
            c0, c1 = tj * tile_n, min((tj + 1) * tile_n, n_kv)
            d0, d1 = c0 // block_n, (c1 - 1) // block_n
            sub = bm[b0:b1 + 1, d0:d1 + 1]
            kept[ti, tj] = bool(sub.any())
            full[ti, tj] = bool(sub.all())
    flag = np.where(full, 0, 1 << 31).astype(np.int64)
    row_ptr = np.zeros(n_ti + 1, dtype=np.int64)
    col_idx = []
    for ti in range(n_ti):
        js = np.nonzero(kept[ti])[0]
        col_idx.extend((js | flag[ti, js]).tolist())
        row_ptr[ti + 1] = row_ptr[ti] + len(js)
    col_ptr = np.zeros(n_tj + 1, dtype=np.int64)
    row_idx = []
    for tj in range(n_tj):
        is_ = np.nonzero(kept[:, tj])[0]
        row_idx.extend((is_ | flag[is_, tj]).tolist())
        col_ptr[tj + 1] = col_ptr[tj] + len(is_)
    as_i32 = lambda a: np.asarray(a, dtype=np.int64).astype(np.uint32).view(np.int32)
    return {
        "row_ptr": row_ptr.astype(np.int32),
        "col_idx": as_i32(col_idx),
        "col_ptr": col_ptr.astype(np.int32),
        "row_idx": as_i32(row_idx),
        "nnz": np.int64(len(col_idx)),
    }


# ---------------------------------------------------------------------------
# Eager attention (floating point: torch on CPU, any float dtype)
# ---------------------------------------------------------------------------


def attention_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      block_mask, softmax_scale: Optional[float] = None,
                      block_m: int = 64, block_n: int = 64,
                      is_causal: bool = False, sink_size: int = 0,
                      window_size: int = 0) -> torch.Tensor:
    """Θ(N²) masked softmax attention, ``sparse_triton_kernel.py:845-902``.

    ``scores = q @ k^T * scale``; entries outside the effective mask get
    ``-inf``; ``softmax`` over keys; rows with no visible key become 0
    through ``nan_to_num``; ``out = probs @ v``.
    """
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(q.shape[-1])
    n_q, n_kv = q.shape[-2], k.shape[-2]
    bm = block_mask.cpu().numpy() if isinstance(block_mask, torch.Tensor) else block_mask
    eff = effective_token_mask(bm, n_q, n_kv, block_m, block_n, is_causal,
                               sink_size, window_size)
    eff_t = torch.from_numpy(np.ascontiguousarray(eff)).to(q.device)
    scores = torch.matmul(q, k.transpose(-2, -1)) * softmax_scale
    scores = scores.masked_fill(~eff_t, float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    probs = torch.nan_to_num(probs, nan=0.0)
    return torch.matmul(probs, v)


def attention_forward_backward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                               do: torch.Tensor, block_mask, **kw
                               ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Forward plus dQ/dK/dV by autograd through :func:`attention_forward`.

    This is the reference's own gradient ground truth: ``benchmark.py``
    compares its kernels against eager autograd (``:322-355``).
    """
    qq = q.detach().clone().requires_grad_(True)
    kk = k.detach().clone().requires_grad_(True)
    vv = v.detach().clone().requires_grad_(True)
    out = attention_forward(qq, kk, vv, block_mask, **kw)
    out.backward(do)
    return out.detach(), qq.grad, kk.grad, vv.grad


def row_lse(q: torch.Tensor, k: torch.Tensor, block_mask, softmax_scale: float,
            block_m: int, block_n: int, is_causal: bool, sink_size: int,
            window_size: int) -> torch.Tensor:
    """Natural-log log-sum-exp per query row, 0 for rows with no visible key.

    The reference kernel stores ``m + log(l)`` with a fully-masked row
    mapped to ``0`` (``sparse_triton_kernel.py:341-352``).
    """
    n_q, n_kv = q.shape[-2], k.shape[-2]
    bm = block_mask.cpu().numpy() if isinstance(block_mask, torch.Tensor) else block_mask
    eff = torch.from_numpy(np.ascontiguousarray(effective_token_mask(
        bm, n_q, n_kv, block_m, block_n, is_causal, sink_size, window_size)))
    scores = torch.matmul(q.double(), k.double().transpose(-2, -1)) * softmax_scale
    scores = scores.masked_fill(~eff, float("-inf"))
    lse = torch.logsumexp(scores, dim=-1)
    return torch.where(torch.isfinite(lse), lse, torch.zeros_like(lse))


def streaming_rows_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           rows, sink: int, window: int, softmax_scale: float
                           ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Exact output and LSE of selected query rows of one (batch, head).

    ``q`` is ``[n_q, D]``, ``k``/``v`` are ``[n_kv, D]`` (any device); rows
    are bottom-right aligned.  Valid for a block mask produced by
    ``make_streaming_mask`` with the same ``sink``/``window`` (its lifted
    mask contains the token mask, so only the token rule matters,
    ``sparse_triton_kernel.py:876-896``).  Computed in float64 over the
    row's visible keys only, so it runs at full benchmark sizes.
    """
    n_q, n_kv = q.shape[0], k.shape[0]
    outs, lses = [], []
    for r in rows:
        qp = n_kv - n_q + int(r)
        keys = torch.arange(0, min(sink, qp + 1), device=k.device)
        lo = max(min(sink, qp + 1), qp - window + 1)
        keys = torch.cat([keys, torch.arange(lo, qp + 1, device=k.device)]) if lo <= qp else keys
        if keys.numel() == 0:
            outs.append(torch.zeros(q.shape[1], dtype=torch.float64, device=q.device))
            lses.append(torch.zeros((), dtype=torch.float64, device=q.device))
            continue
        s = (k[keys].double() @ q[int(r)].double()) * softmax_scale
        lse = torch.logsumexp(s, dim=0)
        p = torch.exp(s - lse)
        outs.append(p @ v[keys].double())
        lses.append(lse)
    return torch.stack(outs), torch.stack(lses)


def visible_key_count(n_q: int, n_kv: int, block_mask, block_m: int, block_n: int,
                      is_causal: bool, sink: int, window: int) -> np.ndarray:
    """Number of visible keys per query row (used by decode byte counts)."""
    bm = block_mask.cpu().numpy() if isinstance(block_mask, torch.Tensor) else block_mask
    return effective_token_mask(bm, n_q, n_kv, block_m, block_n, is_causal,
                                sink, window).sum(axis=1)


def ring_cache_positions(sink: int, window: int, seq_len: int) -> np.ndarray:
    """Position held by each row of a StreamingLLM ring cache after positions
    [0, seq_len) were appended in order (-1 = empty row).  Restates the
    definition: the query at p sees [0, sink) and (p - window, p]
    (upstream token rule, sparse_triton_kernel.py:315-320); row r < sink holds
    position r, position p >= sink the row sink + (p - sink) % window, and a
    later position overwrites an earlier one.  Test infrastructure."""
    rows = np.full(sink + window, -1, dtype=np.int64)
    for p in range(seq_len):
        if p >= sink and window == 0:
            continue  # never visible to a later query
        r = p if p < sink else sink + (p - sink) % window
        rows[r] = p
    return rows
