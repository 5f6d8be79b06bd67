"""The reference's CSV row contracts, kept column for column.

The reference's aggregators and checkers read rows by these exact headers, so
the drivers here can emit them unchanged (``--schema p35`` / ``--schema ref``):

  P35_FIELDS   the 100-field GEMM comparison row, src/gemm/gemm_comparison.py:324-440
  MEM_FIELDS   the 37-column memory-path row, src/memory/ldgsts.cu:741-752
               (tma.cu:1028-1039 prints the same header)
  UMMA_FIELDS  the 37-column UMMA row, src/compute/umma_1sm.cu:976-983

`tests/golden/row_contracts.json` holds the same three headers as extracted from
the reference's own sources by `tests/golden/make_golden.py`; a CPU test pins
these tuples to it. The value conventions follow the reference: a field with no
meaning for the row's method carries ``not_applicable``
(gemm_comparison.py:105-109, 1830-1837); reals are plain fixed-point decimals
with a per-field number of digits (gemm_comparison.py:442-452, 1769-1800).
"""
from __future__ import annotations

import hashlib
import math
import os
import subprocess
from pathlib import Path

NOT_APPLICABLE = "not_applicable"
BOOL_TRUE, BOOL_FALSE = "true", "false"

P35_FIELDS = (
    "schema_version", "experiment", "unit", "run_kind",
    "shape_index", "shape_id", "candidate_index", "method", "variant",
    "m", "n", "k", "l", "ab_dtype", "acc_dtype", "c_dtype", "a_major", "b_major", "c_major",
    "scheduler", "mma_tiler_m", "mma_tiler_n", "cluster_m", "cluster_n", "use_2cta_instrs",
    "use_tma_store", "max_active_clusters",
    "order_a", "order_b", "order_c", "order_d", "transa", "transb", "lda", "ldb", "ldc", "ldd",
    "compute_type", "scale_type", "pointer_mode", "epilogue", "alpha", "beta", "search_mode",
    "workspace_limit_bytes", "workspace_bytes", "alignment_a_bytes", "alignment_b_bytes",
    "alignment_c_bytes", "alignment_d_bytes", "heuristic_requested", "heuristic_returned",
    "heuristic_index", "algo_id", "tile_id", "stages_id", "split_k", "reduction_scheme",
    "cta_swizzling", "custom_option", "inner_shape_id", "cluster_shape_id", "waves_count",
    "cublaslt_version",
    "seed", "reference", "atol", "rtol", "correctness", "max_abs_error", "max_rel_error",
    "compile_time_ms", "setup_time_ms", "first_launch_ms", "kernel_time_ms",
    "warmup_iterations", "iterations", "cache_mode",
    "flop_count", "tflops", "throughput_ratio_vs_cublaslt", "gap_to_cublaslt_pct",
    "rank_within_shape", "best_cutedsl_variant", "is_best_cutedsl",
    "gpu_name", "gpu_uuid", "compute_capability", "driver_version", "cuda_toolkit_version",
    "torch_cuda_version", "cutedsl_version", "cutlass_commit", "operand_factory_sha256",
    "upstream_kernel_file", "upstream_kernel_git_blob", "upstream_kernel_sha256",
    "git_commit", "git_dirty", "publishable",
)

# Fields that carry a value only on a row that runs its own kernel (the
# reference's CuTe DSL rows; here the B200 kernel), and only on a cuBLASLt row
# (gemm_comparison.py:470-526).
KERNEL_ONLY_FIELDS = (
    "scheduler", "mma_tiler_m", "mma_tiler_n", "cluster_m", "cluster_n", "use_2cta_instrs",
    "use_tma_store", "max_active_clusters", "compile_time_ms", "upstream_kernel_file",
    "upstream_kernel_git_blob", "upstream_kernel_sha256",
)
CUBLASLT_ONLY_FIELDS = (
    "order_a", "order_b", "order_c", "order_d", "transa", "transb", "lda", "ldb", "ldc", "ldd",
    "compute_type", "scale_type", "pointer_mode", "epilogue", "alpha", "beta", "search_mode",
    "workspace_limit_bytes", "workspace_bytes", "alignment_a_bytes", "alignment_b_bytes",
    "alignment_c_bytes", "alignment_d_bytes", "heuristic_requested", "heuristic_returned",
    "heuristic_index", "algo_id", "tile_id", "stages_id", "split_k", "reduction_scheme",
    "cta_swizzling", "custom_option", "inner_shape_id", "cluster_shape_id", "waves_count",
    "cublaslt_version", "setup_time_ms",
)

# Digits after the decimal point per kind of real (gemm_comparison.py:442-452).
DECIMALS = {"timing": 6, "error": 9, "tolerance": 9, "scalar": 9, "waves": 6, "tflops": 6,
            "ratio": 9, "gap": 6}
TIMING_FIELDS = ("compile_time_ms", "setup_time_ms", "first_launch_ms", "kernel_time_ms")

# The reference bridge's frozen plan attributes (gemm_comparison.py:155-173) as
# they are written into a cuBLASLt row.
CUBLASLT_FROZEN_TEXT = {
    "order_a": "CUBLASLT_ORDER_ROW", "order_b": "CUBLASLT_ORDER_ROW",
    "order_c": "CUBLASLT_ORDER_ROW", "order_d": "CUBLASLT_ORDER_ROW",
    "transa": "CUBLAS_OP_N", "transb": "CUBLAS_OP_T", "compute_type": "CUBLAS_COMPUTE_32F",
    "scale_type": "CUDA_R_32F", "pointer_mode": "CUBLASLT_POINTER_MODE_HOST",
    "epilogue": "CUBLASLT_EPILOGUE_DEFAULT", "search_mode": "CUBLASLT_SEARCH_BEST_FIT",
    "workspace_limit_bytes": "67108864", "heuristic_requested": "32",
}

MEM_FIELDS = (
    "schema_version", "timestamp_utc", "run_kind", "method", "sample_index", "stages",
    "tile_width_elements", "tile_width_bytes", "tile_height", "stage_bytes",
    "bytes_in_flight_per_sm", "vector_bytes", "copies_per_thread_per_stage",
    "threads_per_cta", "target_ctas_per_sm", "occupancy_ctas_per_sm", "grid_blocks",
    "sm_count", "smem_reservation_bytes", "l2_bytes", "requested_working_set_bytes",
    "working_set_bytes", "working_set_l2_ratio", "passes", "useful_bytes", "warmup_ms",
    "kernel_time_ms", "effective_gbps", "correctness", "mismatches", "gpu_name", "gpu_uuid",
    "compute_capability", "cuda_driver_version", "cuda_runtime_version", "git_commit",
    "git_dirty",
)

UMMA_FIELDS = (
    "schema_version", "timestamp_utc", "run_kind", "publishable", "method", "sample_index",
    "cta_group", "m", "n", "k", "depth", "iterations", "warmup_iterations", "repetitions",
    "umma_per_iteration", "total_umma", "flops_per_umma", "total_flops", "elapsed_cycles",
    "cycles_per_umma", "flops_per_cycle", "threads_per_cta", "grid_blocks", "tmem_columns",
    "operand_path", "input_type", "accumulator_type", "correctness", "mismatches",
    "max_abs_error", "gpu_name", "gpu_uuid", "compute_capability", "cuda_driver_version",
    "cuda_runtime_version", "git_commit", "git_dirty",
)


def format_fixed(value, decimals: int) -> str:
    """A finite real as a plain fixed-point decimal (no exponent); NaN/inf refused."""
    number = float(value)
    if not math.isfinite(number):
        raise ValueError(f"{value!r} is not finite")
    text = f"{number:.{decimals}f}"
    return "0." + "0" * decimals if text.startswith("-") and float(text) == 0.0 else text


def _repo_root() -> Path:
    return Path(__file__).resolve().parents[3]


def _git(args):
    try:
        r = subprocess.run(["git", *args], cwd=_repo_root(), capture_output=True, text=True,
                           timeout=30)
    except (OSError, subprocess.SubprocessError):
        return None
    return r.stdout.strip() if r.returncode == 0 else None


def git_state() -> dict:
    """This repository's commit and dirty flag; `not_available` outside a git checkout
    (e.g. a copy of the tree without .git); B200_GIT_COMMIT overrides the commit."""
    commit = os.environ.get("B200_GIT_COMMIT") or _git(["rev-parse", "HEAD"])
    if not commit:
        return {"git_commit": "not_available", "git_dirty": "not_available"}
    status = _git(["status", "--porcelain", "--untracked-files=no"])
    return {"git_commit": commit,
            "git_dirty": "not_available" if status is None else (BOOL_TRUE if status else BOOL_FALSE)}


def file_identity(path: Path) -> dict:
    """sha256 and git blob id of a source file (the reference's upstream_kernel_* fields)."""
    data = path.read_bytes()
    blob = hashlib.sha1(b"blob %d\0" % len(data) + data).hexdigest()
    return {"sha256": hashlib.sha256(data).hexdigest(), "blob": blob}


def device_provenance(torch, index: int = 0) -> dict:
    """GPU name / UUID / compute capability, driver and runtime versions."""
    props = torch.cuda.get_device_properties(index)
    driver = None
    try:
        import pynvml
        pynvml.nvmlInit()
        driver = pynvml.nvmlSystemGetDriverVersion()
        if isinstance(driver, bytes):
            driver = driver.decode()
        pynvml.nvmlShutdown()
    except Exception:  # noqa: BLE001 - NVML absent: the field says so
        driver = None
    try:
        from .. import _lib
        rt = _lib.device_probe(index)["runtime_version"]
    except Exception:  # noqa: BLE001
        rt = None
    return {"gpu_name": props.name, "gpu_uuid": f"GPU-{props.uuid}",
            "compute_capability": f"{props.major}.{props.minor}",
            "driver_version": driver or "not_available",
            "cuda_runtime_version": str(rt) if rt is not None else "not_available",
            "torch_cuda_version": str(torch.version.cuda)}


def cuda_toolkit_version() -> str:
    try:
        r = subprocess.run(["nvcc", "--version"], capture_output=True, text=True, timeout=30)
    except (OSError, subprocess.SubprocessError):
        return "not_available"
    for tok in r.stdout.replace(",", " ").split():
        if tok.startswith("V") and tok[1:2].isdigit():
            return tok[1:]
    return "not_available"


def cutedsl_version() -> str:
    try:
        import cutlass
        return str(cutlass.__version__)
    except Exception:  # noqa: BLE001
        return NOT_APPLICABLE


def p35_text(row: dict) -> dict:
    """Serialise one GEMM row into the p35 value conventions: every P35 field present,
    reals fixed-point, booleans true/false, missing meaning -> not_applicable."""
    out = {}
    for f in P35_FIELDS:
        v = row.get(f)
        if v is None:
            out[f] = NOT_APPLICABLE
        elif isinstance(v, str):
            out[f] = v
        elif isinstance(v, bool):
            out[f] = BOOL_TRUE if v else BOOL_FALSE
        elif isinstance(v, int):
            out[f] = str(v)
        elif f in TIMING_FIELDS:
            out[f] = format_fixed(v, DECIMALS["timing"])
        elif f in ("max_abs_error", "max_rel_error"):
            out[f] = format_fixed(v, DECIMALS["error"])
        elif f in ("atol", "rtol"):
            out[f] = format_fixed(v, DECIMALS["tolerance"])
        elif f in ("alpha", "beta"):
            out[f] = format_fixed(v, DECIMALS["scalar"])
        elif f == "waves_count":
            out[f] = format_fixed(v, DECIMALS["waves"])
        elif f == "tflops":
            out[f] = format_fixed(v, DECIMALS["tflops"])
        elif f == "throughput_ratio_vs_cublaslt":
            out[f] = format_fixed(v, DECIMALS["ratio"])
        elif f == "gap_to_cublaslt_pct":
            out[f] = f"{float(v):.{DECIMALS['gap']}f}"
        else:
            out[f] = repr(float(v))
    return out
