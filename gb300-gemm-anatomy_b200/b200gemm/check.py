"""Result checks of the drivers (the reference's check path and the product tolerance).

``validate_result`` is the reference's complete-result rule
(src/gemm/gemm_comparison.py:2725-2762): NaN-prefilled output, every element
finite, |D - R| <= atol + rtol*|R| with atol 1e-1, rtol 1e-5, and
max_rel_error with a denominator floor of 1.0.

``bf16_tolerance_check`` is the product rule for bf16 output: relative
Frobenius error <= 1e-2 and, per element,
|D - R| <= ulp_bf16(|R| + eps_acc)/2 + eps_acc, eps_acc = 2^-20 * K * max|a| * max|b|
(bf16 output rounding plus fp32 accumulation-order slack).
"""
from __future__ import annotations

import math

import torch

from ._lib import CorrectnessError

REF_ATOL = 1e-1
REF_RTOL = 1e-5
REL_ERROR_DENOMINATOR_FLOOR = 1.0
REL_FRO_MAX = 1e-2


def validate_result(label: str, reference: torch.Tensor, result: torch.Tensor):
    """Reference rule; returns (max_abs_error, max_rel_error) or raises CorrectnessError."""
    result = result.to(dtype=torch.float32)
    if tuple(result.shape) != tuple(reference.shape):
        raise CorrectnessError(f"{label}: shape {tuple(result.shape)} != {tuple(reference.shape)}")
    if not bool(torch.isfinite(result).all()):
        raise CorrectnessError(f"{label}: the result contains non-finite values (unwritten tiles)")
    diff = (result - reference).abs()
    tolerated = REF_ATOL + REF_RTOL * reference.abs()
    mismatches = int((diff > tolerated).sum().item())
    max_abs = float(diff.max().item()) if diff.numel() else 0.0
    max_rel = float((diff / reference.abs().clamp_min(REL_ERROR_DENOMINATOR_FLOOR)).max().item()) \
        if diff.numel() else 0.0
    if mismatches:
        raise CorrectnessError(f"{label}: {mismatches} element(s) exceed atol={REF_ATOL} "
                               f"rtol={REF_RTOL}; max_abs_error={max_abs} max_rel_error={max_rel}")
    return max_abs, max_rel


def ulp_bf16(x: torch.Tensor) -> torch.Tensor:
    """Spacing of bf16 numbers at |x| (8 significant bits), for |x| >= 2^-126."""
    ax = x.abs().clamp_min(2.0 ** -126)
    return torch.exp2(torch.floor(torch.log2(ax)) - 7.0)


def bf16_tolerance_check(label: str, reference: torch.Tensor, result: torch.Tensor, k: int,
                         max_abs_a: float, max_abs_b: float):
    """Product rule for bf16 output; returns a dict of error statistics or raises."""
    ref = reference.to(torch.float32)
    res = result.to(torch.float32)
    if tuple(res.shape) != tuple(ref.shape):
        raise CorrectnessError(f"{label}: shape {tuple(res.shape)} != {tuple(ref.shape)}")
    if not bool(torch.isfinite(res).all()):
        raise CorrectnessError(f"{label}: the result contains non-finite values (unwritten tiles)")
    eps_acc = 2.0 ** -20 * k * max_abs_a * max_abs_b
    diff = (res - ref).abs()
    tol = ulp_bf16(ref.abs() + eps_acc) / 2 + eps_acc
    bad = int((diff > tol).sum().item())
    ref_norm = float(torch.linalg.vector_norm(ref.double()).item())
    rel_fro = float(torch.linalg.vector_norm((res - ref).double()).item()) / max(ref_norm, 1e-30)
    stats = {"rel_fro": rel_fro, "max_abs_error": float(diff.max().item()) if diff.numel() else 0.0,
             "violations": bad, "eps_acc": eps_acc}
    if bad or not (rel_fro <= REL_FRO_MAX or ref_norm == 0.0) or math.isnan(rel_fro):
        raise CorrectnessError(f"{label}: {bad} element(s) outside bf16 rounding tolerance, "
                               f"rel_fro={rel_fro:.3e}, max_abs={stats['max_abs_error']:.3e}")
    return stats
