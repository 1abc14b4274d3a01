"""ctypes binding to ``libsbfa.so`` (C ABI in ``include/sbfa.h``).

Only plain pointers, integers and floats cross the boundary: tensors are
passed as ``data_ptr()`` and the launch stream as torch's current
``cudaStream_t``.  A nonzero status from the library becomes a
``RuntimeError`` carrying the library's own message.

There is no fallback: if the library is missing, :func:`lib` raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsbfa.so")

F16, BF16, F32, F64 = 0, 1, 2, 3
_DTYPE_CODE = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32, torch.float64: F64}

_lib: Optional[ctypes.CDLL] = None
_lock = threading.Lock()

_i64, _i32, _f64, _vp = ctypes.c_int64, ctypes.c_int, ctypes.c_double, ctypes.c_void_p

_SIGNATURES = {
    "sbfa_abi_version": ([], _i32),
    "sbfa_last_error": ([ctypes.c_char_p, ctypes.c_size_t], _i32),
    "sbfa_device_status": ([ctypes.POINTER(_i32)], _i32),
    "sbfa_launch_count": ([], _i64),
    "sbfa_timing_enable": ([_i32], _i32),
    "sbfa_timing_read": ([_i32, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double),
                          ctypes.POINTER(_i64), ctypes.POINTER(_i32)], _i32),
    "sbfa_streaming_mask": ([_i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp], _i32),
    "sbfa_dense_mask": ([_i64, _i64, _i64, _i64, _i32, _vp, _vp], _i32),
    "sbfa_build_plan": ([_vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp],
                        _i32),
    "sbfa_plan_tiles": ([_i32, _i32, _i64, _i64, ctypes.POINTER(_i64), ctypes.POINTER(_i64)],
                        _i32),
    "sbfa_fwd": ([_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32, _f64, _i32,
                  _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _vp], _i32),
    "sbfa_bwd": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                  _i64, _i32, _f64, _i32, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _vp,
                  _vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp], _i32),
    "sbfa_bwd_workspace_bytes": ([_i64, _i64, _i64, _i32, _i64], _i64),
    "sbfa_bwd_ds_workspace_bytes": ([_i64, _i64, _i64, _i32, _i64], _i64),
    "sbfa_plan_csc_positions": ([_vp, _vp, _vp, _vp, _i64, _vp, _vp], _i32),
    "sbfa_decode": ([_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32, _f64, _i32, _i64,
                     _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _i64, _vp], _i32),
    "sbfa_decode_workspace_bytes": ([_i64, _i64, _i64, _i64, _i64], _i64),
    "sbfa_selftest_wait_timeout": ([_i64, _vp], _i32),
    "sbfa_ring_append": ([_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _i64, _i64, _i64, _i64,
                          _vp], _i32),
    "sbfa_ring_decode": ([_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _f64, _i64, _i64,
                          _i64, _vp, _i64, _vp], _i32),
    "sbfa_ring_decode_workspace_bytes": ([_i64, _i64, _i64, _i64, _i64], _i64),
    "sbfa_decode_supported": ([_i32, _i64], _i32),
    "sbfa_decode_noalloc": ([_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32, _f64, _i32,
                             _i64, _i64, _vp, _i64, _i64, _vp], _i32),
}

EXPORTED = tuple(_SIGNATURES)


def lib() -> ctypes.CDLL:
    """Load ``libsbfa.so`` once (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"libsbfa.so not found at {LIB_PATH}; build it with "
                    "`python graph-kernel-injection_b200/build_native.py` "
                    "(there is no non-CUDA fallback)")
            h = ctypes.CDLL(LIB_PATH)
            for name, (args, res) in _SIGNATURES.items():
                fn = getattr(h, name)
                fn.argtypes = args
                fn.restype = res
            _lib = h
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().sbfa_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"libsbfa {what} failed (status {rc}): {last_error()}")


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}; expected float16, bfloat16, float32 or "
                         "float64") from None


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def device_status() -> int:
    """Read-and-clear the kernels' status word on the current device."""
    out = ctypes.c_int(0)
    check(lib().sbfa_device_status(ctypes.byref(out)), "device_status")
    return out.value


def timing(on: bool) -> None:
    """Enable / disable per-launch CUDA-event timing inside the library."""
    check(lib().sbfa_timing_enable(1 if on else 0), "timing_enable")


def timing_read(max_kernels: int = 64) -> dict:
    """{kernel name: (total ms, launches)} recorded since the last read."""
    names = ctypes.create_string_buffer(64 * max_kernels)
    ms = (ctypes.c_double * max_kernels)()
    cnt = (_i64 * max_kernels)()
    n = _i32(0)
    check(lib().sbfa_timing_read(max_kernels, names, ms, cnt, ctypes.byref(n)), "timing_read")
    out = {}
    for i in range(n.value):
        nm = names.raw[64 * i:64 * (i + 1)].split(b"\0", 1)[0].decode()
        out[nm] = (float(ms[i]), int(cnt[i]))
    return out


def launch_count() -> int:
    return int(lib().sbfa_launch_count())


def plan_tiles(pass_id: int, dtype: torch.dtype, head_dim: int, n_q: int):
    tm, tn = ctypes.c_int64(0), ctypes.c_int64(0)
    check(lib().sbfa_plan_tiles(pass_id, dtype_code(dtype), head_dim, n_q,
                                ctypes.byref(tm), ctypes.byref(tn)), "plan_tiles")
    return int(tm.value), int(tn.value)
