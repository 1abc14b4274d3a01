"""Tolerance checks shared by the GPU parity tests.

float16 / bfloat16 results are held to the fixed bounds the north-star
bar states, against a float64 (or float32, at full size) oracle on the
same rounded inputs: max-abs error <= 2e-2 and relative L2 error <= 5e-3.
The max-abs bound applies to the computation: each element may in addition
differ from the exact value by half a unit in the last place of the output
type at that value (the error of storing the exact result as a 16-bit
number, which no kernel can avoid: 2^-9 |x| for bfloat16, 2^-12 |x| for
float16, e.g. up to 0.0156 for a bfloat16 result in [4, 8)).  The bound is
never scaled by the reference's magnitude otherwise.

Every check prints its measured errors (the raw max-abs and the max-abs
beyond the output rounding); with SBFA_PARITY_LOG set to a file path each
one is also appended there as a JSON line, so a GPU run leaves the full
table of measured errors behind.
"""

from __future__ import annotations

import json
import os

import torch

MAX_ABS = 2e-2
REL_L2 = 5e-3


def _log(label: str, dtype, err: float, beyond: float, rel: float, ref_max: float) -> None:
    test = os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0]
    print(f"parity {test} {label} {dtype}: max-abs {err:.3e} (beyond output rounding "
          f"{beyond:.3e}) rel-L2 {rel:.3e} max|ref| {ref_max:.3e}")
    path = os.environ.get("SBFA_PARITY_LOG")
    if path:
        with open(path, "a") as fh:
            fh.write(json.dumps({"test": test, "tensor": label, "dtype": str(dtype),
                                 "max_abs": err, "max_abs_beyond_rounding": beyond,
                                 "rel_l2": rel, "ref_max": ref_max}) + "\n")


def half_ulp(ref: torch.Tensor, dtype) -> torch.Tensor:
    """Half a unit in the last place of `dtype` at each |ref| (0 for
    float32 / float64 results, whose rounding is far below the bounds)."""
    bits = {torch.bfloat16: 8, torch.float16: 11}.get(dtype)
    if bits is None:
        return torch.zeros_like(ref)
    _, e = torch.frexp(ref)            # |ref| in [2^(e-1), 2^e)
    return torch.ldexp(torch.ones_like(ref), e - 1 - bits)


def errors(got: torch.Tensor, ref: torch.Tensor):
    got, ref = got.double().cpu(), ref.double().cpu()
    err = (got - ref).abs().max().item() if got.numel() else 0.0
    rel = ((got - ref).norm() / ref.norm().clamp_min(1e-30)).item()
    return err, rel, (ref.abs().max().item() if ref.numel() else 0.0)


def check_half(got: torch.Tensor, ref: torch.Tensor, dtype=torch.bfloat16,
               label: str = "") -> None:
    """16-bit result against a high-precision oracle: fixed max-abs and
    rel-L2 bounds (not scaled by the reference's magnitude)."""
    assert torch.isfinite(got).all(), f"{label}: non-finite output"
    err, rel, ref_max = errors(got, ref)
    g64, r64 = got.double().cpu(), ref.double().cpu()
    beyond = ((g64 - r64).abs() - half_ulp(r64, dtype)).max().item() if got.numel() else 0.0
    _log(label, dtype, err, beyond, rel, ref_max)
    assert beyond <= MAX_ABS, (f"{label}: max-abs {err:.3e}, {beyond:.3e} beyond the output "
                               f"rounding > {MAX_ABS} (max|ref| {ref_max:.3g})")
    assert rel <= REL_L2, f"{label}: rel-L2 {rel:.3e} > {REL_L2}"
