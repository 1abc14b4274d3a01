"""Generate golden fixtures by running the upstream reference itself.

Usage::

    python tests/golden/make_golden.py <path-to-upstream-checkout>

The upstream project (Hridambiswas/graph-kernel-injection) is pure
Python + torch, so its ``sparse_triton_kernel.py`` imports on a CPU-only
host (the Triton kernels are never launched here).  This script loads
that file under a private module name and records, for every shape its
own tests use plus the five benchmark configurations:

* ``block_masks.npz`` - ``make_streaming_mask`` (ref ``:104-181``) and
  ``make_dense_mask`` (ref ``:184-210``) outputs, bit-packed;
* ``token_masks.json`` - ``streaming_token_mask`` (ref ``:905-932``)
  popcount, per-row counts and a SHA-256 of the packed bits;
* ``attention_cases.npz`` - ``reference_block_sparse_attention``
  (ref ``:845-902``) outputs and autograd dQ/dK/dV in float64 on seeded
  inputs (the inputs are stored too, so no RNG agreement is assumed);
* ``attention_tc_cases.npz`` - the same for inputs rounded to bfloat16 /
  float16 at head_dim 128 / 64 with 128 x 128 blocks, the shapes the
  tensor-core kernels take (``--tc-only`` regenerates just this file).

The fixtures are committed; the GPU box never needs the upstream tree.
"""

from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (n_q, n_kv, sink, window, block_m, block_n).  Sources: upstream
# tests/test_streaming_definition.py:106-118 and :228-236,
# tests/test_mask_equivalence.py:310-321, tests/test_oracle.py:29-37,
# and the five benchmark configurations.
BLOCK_CASES = [
    (1, 1000, 4, 256, 1, 64), (1, 1023, 4, 256, 1, 64), (1, 1025, 4, 256, 1, 64),
    (16, 1000, 4, 128, 16, 64), (1000, 1000, 4, 128, 64, 64),
    (1023, 1023, 4, 128, 64, 64), (1025, 1025, 4, 128, 64, 64),
    (4, 10, 8, 4, 2, 2), (16, 16, 4, 8, 8, 8), (128, 1024, 4, 128, 16, 64),
    (32, 32, 4, 8, 8, 8), (4, 32, 4, 8, 2, 8), (1, 32, 4, 8, 1, 8),
    (64, 64, 4, 16, 16, 16), (64, 128, 4, 32, 16, 32), (128, 128, 8, 32, 32, 32),
    (256, 256, 4, 64, 64, 64), (128, 1024, 4, 128, 64, 64),
    (64, 64, 0, 64, 16, 16), (64, 64, 64, 0, 16, 16),
    # benchmark configurations
    (1024, 1024, 4, 256, 64, 64),            # cfg1
    (16384, 16384, 4, 2048, 128, 128),       # cfg2
    (131072, 131072, 4, 4096, 128, 128),     # cfg3
    (1, 100001, 4, 2048, 1, 64),             # cfg4 (decode, BM clamped to 1)
    (32768, 32768, 4, 2048, 64, 64),         # cfg5, injector default tiles
    (32768, 32768, 4, 2048, 128, 128),       # cfg5 with 128 tiles
    # extra edge cases for the GPU plan builder
    (1, 1, 0, 0, 1, 1), (7, 300, 0, 5, 3, 17), (300, 7, 2, 1, 17, 3),
    (129, 257, 1, 64, 128, 128), (255, 255, 4, 64, 128, 64),
]

DENSE_CASES = [  # (n_q, n_kv, block_m, block_n, causal)
    (64, 64, 16, 16, False), (64, 64, 16, 16, True), (256, 128, 64, 32, True),
    (1024, 1024, 128, 128, True),
]

TOKEN_CASES = [  # upstream tests/test_streaming_definition.py:76-101
    (1, 1000, 4, 256), (1, 1000, 0, 256), (1, 1000, 4, 0), (1, 1000, 4, 2048),
    (16, 16, 4, 8), (64, 64, 4, 16), (2, 10, 4, 4), (1000, 1000, 4, 128),
    (1023, 1023, 4, 128), (1025, 1025, 4, 128), (4, 10, 8, 4), (16, 1000, 4, 128),
    (128, 1024, 4, 128), (4, 4, 4, 1),
]

# Attention cases: (name, B, H, n_q, n_kv, D, bm, bn, is_causal, S, W, mask_kind)
ATTN_CASES = [
    ("gradcheck_tiny", 1, 2, 64, 64, 16, 16, 16, True, 4, 16, "streaming"),
    ("bottom_right", 1, 1, 16, 500, 16, 16, 64, True, 4, 128, "streaming"),
    ("decode", 2, 1, 1, 600, 16, 1, 64, True, 4, 256, "streaming"),
    ("ragged", 1, 1, 515, 515, 8, 64, 64, True, 4, 128, "streaming"),
    ("small_q_big_sink", 1, 2, 4, 10, 8, 2, 2, True, 8, 4, "streaming"),
    ("window_only", 1, 2, 64, 64, 16, 16, 16, True, 0, 64, "streaming"),
    ("custom_empty_row", 1, 2, 32, 32, 16, 16, 16, False, 0, 0, "custom_empty_row"),
    ("custom_causal", 1, 1, 96, 160, 16, 32, 32, True, 4, 48, "custom_random"),
]


# Cases that reach the tensor-core kernels (float16 / bfloat16, head_dim 64 or
# 128, BM = BN = 128): (name, B, H, n_q, n_kv, D, bm, bn, is_causal, S, W,
# mask_kind, dtype).  Inputs are drawn in float64, rounded to the 16-bit type
# and stored as that type's bit patterns; the upstream reference runs in
# float64 on the rounded values and its outputs are stored as float32.
ATTN_TC_CASES = [
    ("tc_bf16_streaming_d128", 1, 1, 384, 384, 128, 128, 128, True, 4, 160, "streaming",
     "bfloat16"),
    ("tc_fp16_bottom_right_d64", 1, 1, 200, 456, 64, 128, 128, True, 4, 200, "streaming",
     "float16"),
    ("tc_fp16_custom_noncausal_d128", 1, 1, 256, 256, 128, 128, 128, False, 0, 0,
     "custom_antidiagonal", "float16"),
]


def load_upstream(root: str):
    path = os.path.join(root, "sparse_triton_kernel.py")
    spec = importlib.util.spec_from_file_location("_upstream_sparse_kernel", path)
    mod = importlib.util.module_from_spec(spec)
    sys.dont_write_bytecode = True
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def key_block(c) -> str:
    return "blk_" + "_".join(str(x) for x in c)


def main(root: str) -> None:
    up = load_upstream(root)
    out = {}
    for c in BLOCK_CASES:
        n_q, n_kv, s, w, bm, bn = c
        m = up.make_streaming_mask(n_q, n_kv, up.StreamingMaskSpec(s, w), bm, bn,
                                   device="cpu").numpy()
        assert m.dtype == np.int32
        out[key_block(c) + "_shape"] = np.array(m.shape, dtype=np.int64)
        out[key_block(c) + "_bits"] = np.packbits(m.astype(bool).ravel())
        out[key_block(c) + "_nnz"] = np.int64(m.sum())
    for c in DENSE_CASES:
        n_q, n_kv, bm, bn, causal = c
        m = up.make_dense_mask(n_q, n_kv, bm, bn, causal=causal, device="cpu").numpy()
        k = "dense_" + "_".join(str(int(x)) for x in c)
        out[k + "_shape"] = np.array(m.shape, dtype=np.int64)
        out[k + "_bits"] = np.packbits(m.astype(bool).ravel())
    np.savez_compressed(os.path.join(HERE, "block_masks.npz"), **out)

    tok = {}
    for c in TOKEN_CASES:
        n_q, n_kv, s, w = c
        m = up.streaming_token_mask(n_q, n_kv, s, w, device="cpu").numpy()
        tok["_".join(str(x) for x in c)] = {
            "popcount": int(m.sum()),
            "row_counts_sha256": hashlib.sha256(
                m.sum(axis=1).astype(np.int64).tobytes()).hexdigest(),
            "bits_sha256": hashlib.sha256(np.packbits(m.ravel()).tobytes()).hexdigest(),
        }
    with open(os.path.join(HERE, "token_masks.json"), "w") as fh:
        json.dump(tok, fh, indent=1, sort_keys=True)

    att = {}
    for (name, B, H, n_q, n_kv, D, bm, bn, causal, s, w, kind) in ATTN_CASES:
        g = torch.Generator().manual_seed(1234)
        q = torch.randn(B, H, n_q, D, generator=g, dtype=torch.float64)
        k = torch.randn(B, H, n_kv, D, generator=g, dtype=torch.float64)
        v = torch.randn(B, H, n_kv, D, generator=g, dtype=torch.float64)
        do = torch.randn(B, H, n_q, D, generator=g, dtype=torch.float64)
        n_qb, n_kb = -(-n_q // bm), -(-n_kv // bn)
        if kind == "streaming":
            mask = up.make_streaming_mask(n_q, n_kv, up.StreamingMaskSpec(s, w), bm, bn,
                                          device="cpu")
        elif kind == "custom_empty_row":
            # upstream tests/test_fully_masked_row.py:149-152
            mask = torch.zeros((n_qb, n_kb), dtype=torch.int32)
            mask[1, 1] = 1
        else:
            mask = (torch.rand(n_qb, n_kb, generator=g) < 0.5).to(torch.int32)
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        o = up.reference_block_sparse_attention(
            qq, kk, vv, mask, block_m=bm, block_n=bn, is_causal=causal,
            sink_size=s, window_size=w)
        o.backward(do)
        p = f"{name}__"
        att[p + "params"] = np.array([B, H, n_q, n_kv, D, bm, bn, int(causal), s, w],
                                     dtype=np.int64)
        att[p + "mask"] = mask.numpy().astype(np.int32)
        for nm, t in (("q", q), ("k", k), ("v", v), ("do", do), ("o", o.detach()),
                      ("dq", qq.grad), ("dk", kk.grad), ("dv", vv.grad)):
            att[p + nm] = t.numpy()
    np.savez_compressed(os.path.join(HERE, "attention_cases.npz"), **att)
    main_tc(up)
    print("wrote", sorted(os.listdir(HERE)))


def main_tc(up) -> None:
    """attention_tc_cases.npz: ATTN_TC_CASES through the upstream reference."""
    att = {}
    for (name, B, H, n_q, n_kv, D, bm, bn, causal, s, w, kind, dt) in ATTN_TC_CASES:
        tdt = getattr(torch, dt)
        g = torch.Generator().manual_seed(4321)
        ins = [torch.randn(B, H, n, D, generator=g, dtype=torch.float64).to(tdt)
               for n in (n_q, n_kv, n_kv, n_q)]
        q, k, v, do = (t.double() for t in ins)
        n_qb, n_kb = -(-n_q // bm), -(-n_kv // bn)
        if kind == "streaming":
            mask = up.make_streaming_mask(n_q, n_kv, up.StreamingMaskSpec(s, w), bm, bn,
                                          device="cpu")
        else:  # row block i keeps only key block n_kb - 1 - i: every 256-row
            # forward tile then holds two partial tiles
            mask = torch.zeros((n_qb, n_kb), dtype=torch.int32)
            for i in range(n_qb):
                mask[i, n_kb - 1 - i] = 1
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        o = up.reference_block_sparse_attention(
            qq, kk, vv, mask, block_m=bm, block_n=bn, is_causal=causal,
            sink_size=s, window_size=w)
        o.backward(do)
        p = f"{name}__"
        att[p + "params"] = np.array([B, H, n_q, n_kv, D, bm, bn, int(causal), s, w],
                                     dtype=np.int64)
        att[p + "dtype"] = np.array(dt)
        att[p + "mask"] = mask.numpy().astype(np.int32)
        for nm, t in zip(("q", "k", "v", "do"), ins):
            att[p + nm] = t.view(torch.int16).numpy()
        for nm, t in (("o", o.detach()), ("dq", qq.grad), ("dk", kk.grad), ("dv", vv.grad)):
            att[p + nm] = t.float().numpy()
    np.savez_compressed(os.path.join(HERE, "attention_tc_cases.npz"), **att)


if __name__ == "__main__":
    if len(sys.argv) not in (2, 3) or (len(sys.argv) == 3 and sys.argv[2] != "--tc-only"):
        raise SystemExit("usage: make_golden.py <upstream checkout> [--tc-only]")
    if len(sys.argv) == 3:
        main_tc(load_upstream(sys.argv[1]))
    else:
        main(sys.argv[1])
