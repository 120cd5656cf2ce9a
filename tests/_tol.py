"""Tolerances of the parity tests, stated once.

Metric 1 (the reference's, tests/test_correctness.py:10-11): norm-wise relative error
    ||y - ref|| / ||ref||, against an fp64 product of the same inputs.
Metric 2 (per element, component-wise): |y - ref| <= RTOL * (|x| @ |w| + |bias|), elementwise.
    This is the relative error of each output measured against the magnitude of its own terms
    (the standard dot-product error bound); a plain |y - ref| / |ref| is unbounded for outputs that
    cancel to near zero.

Bounds (relative error <= 1e-3 vs fp64 on the GEMM path, <= 1e-5 on the
skinny fp32-accumulate path, no inf/NaN):
    GEMM path (M > 8), any output dtype:  norm 1e-3, component-wise 1e-3
    skinny path (M <= 8), fp32 output:    norm 1e-5, component-wise 1e-5
    skinny path (M <= 8), fp16 output:    norm 1e-3, component-wise 1e-3 (fp16 output rounding alone
                                          is up to 2^-11 = 4.9e-4 of |y|)
On the GEMM path fp32 activations are rounded to fp16 (as in the reference), which alone costs
up to 2^-11 of |x|@|w|; fp16 output rounding adds up to 2^-11 of |y|.
"""
from __future__ import annotations

import torch

GEMM_NORM = GEMM_RTOL = 1e-3
SKINNY_NORM = SKINNY_RTOL = 1e-5


def rel_err(y: torch.Tensor, ref: torch.Tensor) -> float:
    ref = ref.double()
    return ((y.double() - ref).norm() / ref.norm().clamp_min(1e-300)).item()


def ref64(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    y = x.double() @ w.double()
    return y + b.double() if b is not None else y


def magnitude64(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    y = x.double().abs() @ w.double().abs()
    return y + b.double().abs() if b is not None else y


def bounds(M: int, out_dtype: torch.dtype) -> tuple[float, float]:
    if M <= 8 and out_dtype == torch.float32:
        return SKINNY_NORM, SKINNY_RTOL
    return GEMM_NORM, GEMM_RTOL


def componentwise_err(y: torch.Tensor, ref: torch.Tensor, mag: torch.Tensor) -> float:
    d = (y.double() - ref.double()).abs()
    return (d / mag.clamp_min(1e-300)).max().item() if d.numel() else 0.0


def assert_close_fp64(y: torch.Tensor, x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None, out_dtype,
                      what: str = "", ref: torch.Tensor | None = None) -> float:
    """Check y against the fp64 product of (x, w, b) with both metrics; returns the norm-wise error."""
    M = x.shape[0]
    norm, rtol = bounds(M, out_dtype)
    assert torch.isfinite(y).all(), f"{what}: non-finite output"
    ref = ref64(x, w, b) if ref is None else ref
    e = rel_err(y, ref)
    assert e <= norm, f"{what}: norm-wise rel err {e:.3e} > {norm:.0e}"
    c = componentwise_err(y, ref, magnitude64(x, w, b))
    assert c <= rtol, f"{what}: component-wise rel err {c:.3e} > {rtol:.0e}"
    return e
