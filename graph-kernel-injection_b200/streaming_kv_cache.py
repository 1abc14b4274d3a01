"""StreamingLLM ring-buffer KV cache for the decode step.

No upstream counterpart: upstream decodes through its prefill kernel with
``N_Q = 1`` over the whole cache (``benchmark.py:799-804``), although the
StreamingLLM rule lets the query at position ``p`` see only positions
``[0, sink)`` and ``(p - window, p]``.  This cache keeps exactly those
``sink + window`` rows per (batch, head): row ``r < sink`` holds position
``r``; position ``p >= sink`` lives in row ``sink + (p - sink) % window``.
Decoding over it gives the same attention as the block-sparse decode over a
full-length cache (``block_sparse_attention`` with ``N_Q == 1``, causal,
``block_m = 1``), with ``(sink + window) / n_kv`` of the memory.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

import sbfa_native as native


class StreamingKVCache:
    """Per-layer K/V ring cache, ``[B, H, sink + window, D]`` each, on one
    CUDA device.  ``append`` adds tokens in order; ``attend`` decodes the
    query of the last appended position."""

    def __init__(self, batch: int, heads: int, head_dim: int, sink_size: int, window_size: int,
                 dtype: torch.dtype = torch.float16, device: str | torch.device = "cuda") -> None:
        if min(batch, heads, head_dim) <= 0:
            raise ValueError("batch, heads and head_dim must be positive")
        if sink_size < 0 or window_size < 0 or sink_size + window_size <= 0:
            raise ValueError("sink_size and window_size must be non-negative, not both zero")
        native.dtype_code(dtype)
        self.batch, self.heads, self.head_dim = batch, heads, head_dim
        self.sink_size, self.window_size = sink_size, window_size
        self.dtype = dtype
        dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        rows = sink_size + window_size
        self.k = torch.zeros(batch, heads, rows, head_dim, dtype=dtype, device=self.device)
        self.v = torch.zeros_like(self.k)
        self.length = 0
        ws = int(native.lib().sbfa_ring_decode_workspace_bytes(batch, heads, head_dim, sink_size,
                                                               window_size))
        self._ws = torch.empty(max(ws, 16), dtype=torch.uint8, device=self.device)

    @property
    def memory_bytes(self) -> int:
        return 2 * self.k.numel() * self.k.element_size()

    def _check(self, t: torch.Tensor, n: Optional[int], name: str) -> torch.Tensor:
        want = (self.batch, self.heads) + ((n,) if n is not None else (t.shape[2],)) + (
            self.head_dim,)
        if t.dim() != 4 or tuple(t.shape) != want:
            raise ValueError(f"{name} must have shape {want}, got {tuple(t.shape)}")
        if t.device != self.device or t.dtype != self.dtype:
            raise ValueError(f"{name} must be {self.dtype} on {self.device}")
        return t.contiguous()

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor) -> None:
        """Append K/V of the next ``k_new.shape[2]`` positions ([B, H, t, D])."""
        k_new = self._check(k_new, None, "k_new")
        v_new = self._check(v_new, k_new.shape[2], "v_new")
        n = k_new.shape[2]
        with torch.cuda.device(self.device):
            native.check(native.lib().sbfa_ring_append(
                self.k.data_ptr(), self.v.data_ptr(), k_new.data_ptr(), v_new.data_ptr(),
                self.batch, self.heads, self.head_dim, native.dtype_code(self.dtype),
                self.sink_size, self.window_size, self.length, n,
                native.stream_ptr(self.device)), "ring_append")
        self.length += n

    def attend(self, q: torch.Tensor, softmax_scale: Optional[float] = None,
               return_lse: bool = False):
        """Attention of the query at position ``length - 1`` ([B, H, 1, D])
        over the cached sink and window; returns O ([B, H, 1, D]) and, with
        ``return_lse``, the natural-log LSE ([B, H, 1] fp32)."""
        if self.length == 0:
            raise RuntimeError("the cache is empty: append the query's own token first")
        q = self._check(q, 1, "q")
        scale = 1.0 / math.sqrt(self.head_dim) if softmax_scale is None else float(softmax_scale)
        o = torch.empty_like(q)
        lse = torch.empty(self.batch, self.heads, 1, dtype=torch.float32, device=self.device)
        with torch.cuda.device(self.device):
            native.check(native.lib().sbfa_ring_decode(
                q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                self.batch, self.heads, self.head_dim, native.dtype_code(self.dtype), scale,
                self.sink_size, self.window_size, self.length, self._ws.data_ptr(),
                self._ws.numel(), native.stream_ptr(self.device)), "ring_decode")
        return (o, lse) if return_lse else o
