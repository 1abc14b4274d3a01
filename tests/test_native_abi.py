"""The C ABI library loads on a CPU-only host and exports exactly what
include/sbfa.h declares; argument validation runs without a GPU."""

from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

import sbfa_native as native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "sbfa.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(sbfa_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(native.LIB_PATH):
        pytest.fail("libsbfa.so is not built (run __graft_entry__.build())")
    return native.lib()


def test_header_and_binding_agree():
    assert declared_functions() == sorted(native.EXPORTED)


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", native.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (sbfa_[a-z0-9_]+)", out))
    missing = set(declared_functions()) - exported
    assert not missing, missing
    for name in declared_functions():
        assert hasattr(lib, name)


def test_abi_version(lib):
    assert lib.sbfa_abi_version() == 5


def test_validation_errors_without_gpu(lib):
    rc = lib.sbfa_streaming_mask(0, 10, 1, 1, 1, 1, None, None)
    assert rc == 1 and "positive" in native.last_error()
    rc = lib.sbfa_streaming_mask(4, 10, -1, 1, 1, 1, None, None)
    assert rc == 1 and "non-negative" in native.last_error()
    rc = lib.sbfa_dense_mask(10, 10, 3, 2, 0, None, None)
    assert rc == 1 and "divide" in native.last_error()
    rc = lib.sbfa_build_plan(None, 4, 4, 1, 1, 1, 1, None, None, None, None, None, None)
    assert rc == 1 and "block_mask" in native.last_error()
    rc = lib.sbfa_fwd(None, None, None, None, None, 1, 1, 0, 4, 16, 0, 1.0, 1, 0, 0, None,
                      16, 16, None, None, None, 0, None)
    assert rc == 1
    rc = lib.sbfa_fwd(None, None, None, None, None, 1, 1, 4, 4, 16, 9, 1.0, 1, 0, 0, None,
                      16, 16, None, None, None, 0, None)
    assert rc == 1 and "dtype" in native.last_error()


def test_plan_tiles_and_decode_support(lib):
    assert native.plan_tiles(3, __import__("torch").float16, 128, 1) == (1, 64)
    tm, tn = native.plan_tiles(0, __import__("torch").float32, 64, 1024)
    assert tm > 0 and tn > 0
    assert lib.sbfa_decode_supported(native.F16, 128) == 1
    assert lib.sbfa_decode_supported(native.F64, 128) == 0
    assert lib.sbfa_decode_supported(native.F16, 24) == 0
    assert lib.sbfa_decode_workspace_bytes(64, 32, 100001, 128, 64) >= 0


def test_last_error_truncates(lib):
    lib.sbfa_streaming_mask(0, 10, 1, 1, 1, 1, None, None)
    buf = ctypes.create_string_buffer(4)
    n = lib.sbfa_last_error(buf, 4)
    assert n > 3 and len(buf.value) == 3


def test_bwd_workspace_bytes(lib):
    """Split scratch is only needed with grouped K/V heads on the
    tensor-core path: one fp32 [dV | dK] 128 x D partial per query head."""
    assert lib.sbfa_bwd_workspace_bytes(4, 32, 128, native.BF16, 32) == 0
    assert lib.sbfa_bwd_workspace_bytes(4, 32, 128, native.BF16, 0) == 0
    assert lib.sbfa_bwd_workspace_bytes(4, 32, 128, native.BF16, 4) == 4 * 32 * 2 * 128 * 128 * 4
    assert lib.sbfa_bwd_workspace_bytes(1, 8, 64, native.F16, 1) == 8 * 2 * 128 * 64 * 4
    assert lib.sbfa_bwd_workspace_bytes(1, 8, 64, native.F32, 1) == 0
    assert lib.sbfa_bwd_workspace_bytes(1, 8, 128, native.BF16, 3) == 0   # 8 % 3 != 0


def test_bwd_ds_workspace_bytes(lib):
    """Stored-dS scratch: B * H * nnz tiles of 128 x 128 16-bit values for
    fp16/bf16 at head_dim 128; 0 elsewhere and when the tile count reaches
    2^31 (TMA coordinates are 32-bit)."""
    assert lib.sbfa_bwd_ds_workspace_bytes(4, 32, 128, native.BF16, 2151) == \
        4 * 32 * 2151 * 128 * 128 * 2
    assert lib.sbfa_bwd_ds_workspace_bytes(1, 2, 128, native.F16, 7) == 2 * 7 * 128 * 128 * 2
    assert lib.sbfa_bwd_ds_workspace_bytes(4, 32, 64, native.BF16, 2151) == 0
    assert lib.sbfa_bwd_ds_workspace_bytes(4, 32, 128, native.F32, 2151) == 0
    assert lib.sbfa_bwd_ds_workspace_bytes(4, 32, 128, native.BF16, 0) == 0
    assert lib.sbfa_bwd_ds_workspace_bytes(1 << 12, 1 << 10, 128, native.BF16, 1 << 9) == 0


def test_debug_library_exports_the_same_symbols():
    """libsbfa_debug.so (device-side bounds checks) is a drop-in build of the
    same ABI."""
    path = os.path.join(os.path.dirname(native.LIB_PATH), "libsbfa_debug.so")
    if not os.path.exists(path):
        pytest.fail("libsbfa_debug.so is not built (run __graft_entry__.build())")
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (sbfa_[a-z0-9_]+)", out))
    assert set(declared_functions()) <= exported
