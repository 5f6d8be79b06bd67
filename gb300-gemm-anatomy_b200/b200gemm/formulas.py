"""Pure arithmetic of the reported metrics (no GPU, no I/O, no state).

Definitions follow the reference study so rows stay comparable:
  flop_count = 2*M*N*K                      (src/gemm/gemm_comparison.py:1626-1641)
  tflops     = flop_count / (ms * 1e9)      (gemm_comparison.py:1644-1662)
  ratio/gap vs a baseline                   (gemm_comparison.py:1665-1763)
  effective_gbps = useful_bytes / s / 1e9   (src/memory/ldgsts.cu:898,913-916)
  umma flop  = 2*M*N*16*depth*iterations    (src/compute/umma_1sm.cu:1164-1167)
  HBM classification of ncu dram bytes      (scripts/analyze_exp01_memory_paths_p14.py:131-141)
"""
from __future__ import annotations

import math

FLOPS_PER_MAC = 2
UMMA_K = 16


class FormulaError(ValueError):
    pass


def _positive_int(name, value):
    if isinstance(value, bool) or not isinstance(value, int) or value <= 0:
        raise FormulaError(f"{name}={value!r} must be a positive integer")
    return value


def _positive_float(name, value):
    v = float(value)
    if not math.isfinite(v) or v <= 0.0:
        raise FormulaError(f"{name}={value!r} must be finite and strictly positive")
    return v


def compute_flop_count(m: int, n: int, k: int) -> int:
    """Exact FLOP count of one GEMM, as a Python int."""
    return FLOPS_PER_MAC * _positive_int("m", m) * _positive_int("n", n) * _positive_int("k", k)


def compute_tflops(flop_count: int, kernel_time_ms: float) -> float:
    """TFLOP/s from an exact FLOP count and a per-launch time in ms."""
    _positive_int("flop_count", flop_count)
    return flop_count / (_positive_float("kernel_time_ms", kernel_time_ms) * 1e9)


def compute_ratio_and_gap(candidate_tflops: float, baseline_tflops: float):
    """(throughput ratio, gap %) of a candidate against a baseline; gap > 0 = slower."""
    ratio = _positive_float("candidate_tflops", candidate_tflops) / _positive_float(
        "baseline_tflops", baseline_tflops)
    return ratio, 100.0 * (1.0 - ratio)


def effective_gbps(useful_bytes: int, kernel_time_ms: float) -> float:
    _positive_int("useful_bytes", useful_bytes)
    return useful_bytes / (_positive_float("kernel_time_ms", kernel_time_ms) / 1e3) / 1e9


def umma_flop_count(m: int, n: int, depth: int, iterations: int) -> int:
    return FLOPS_PER_MAC * _positive_int("m", m) * _positive_int("n", n) * UMMA_K * \
        _positive_int("depth", depth) * _positive_int("iterations", iterations)


def flops_per_cycle_per_sm(flop_count: int, cycles: int, sms: int) -> float:
    return _positive_int("flop_count", flop_count) / _positive_int("cycles", cycles) / \
        _positive_int("sms", sms)


def roofline_fraction(achieved: float, peak: float) -> float:
    return _positive_float("achieved", achieved) / _positive_float("peak", peak)


HBM_VALIDATED_MIN_RATIO = 0.90
READ_AMPLIFICATION_MAX_RATIO = 1.10


def classify_hbm(dram_read_bytes, useful_bytes):
    """(classification, flags, ratio) of the reference's HBM evidence rule.

    Same thresholds and outcomes as classify_hbm in
    scripts/analyze_exp01_memory_paths_p14.py:1887-1903: below 0.90 of the
    useful bytes is INCONCLUSIVE, above 1.10 is validated with a
    READ_AMPLIFICATION flag.
    """
    if dram_read_bytes is None:
        return "INCONCLUSIVE", ["DRAM_READ_METRIC_UNAVAILABLE"], None
    if not math.isfinite(dram_read_bytes) or dram_read_bytes < 0:
        return "INCONCLUSIVE", ["DRAM_READ_BYTES_MALFORMED"], None
    if not math.isfinite(useful_bytes) or useful_bytes <= 0:
        return "INCONCLUSIVE", ["USEFUL_BYTES_MALFORMED"], None
    ratio = dram_read_bytes / useful_bytes
    if ratio < HBM_VALIDATED_MIN_RATIO:
        return "INCONCLUSIVE", ["RATIO_BELOW_THRESHOLD"], ratio
    if ratio > READ_AMPLIFICATION_MAX_RATIO:
        return "HBM_VALIDATED", ["READ_AMPLIFICATION"], ratio
    return "HBM_VALIDATED", [], ratio
