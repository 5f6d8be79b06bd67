"""GEMM comparison driver: the reference's P3.5 driver shape with the B200 kernel as candidate.

Same command-line contract as src/gemm/gemm_comparison.py (build_arg_parser,
:3280-3332): --warmup-iterations [1..100] (default 5), --iterations [1..100]
(default 20), --self-test (GPU-free), CSV on stdout only after every row
passed its correctness check, diagnostics on stderr, exit 0 / 1 (failure) /
2 (usage). Per shape: operands built once outside every timer, output
NaN-prefilled before each candidate, correctness before timing, CUDA-event
steady state over `iterations` launches (gemm_comparison.py:3055-3074).

Additions for B200: --shapes picks the shape set (the reference's five frozen
shapes by default; also the benchmark configs c1/c4/c5), --operands picks the
reference's integer operands (seed 1111, exact fp32 results) or the configs'
seeded distributions, --out-dtype f32 (reference contract) or bf16, and the
candidates are the B200 persistent 1-CTA and 2-CTA kernels plus cuBLAS
(torch.matmul) as a context baseline.
"""
from __future__ import annotations

import argparse
import io
import math
import sys

from . import row_contracts

SCHEMA_VERSION = "b200.p35.1"
EXPERIMENT = "gemm_comparison"
UNIT = "b200_gemm"
DEFAULT_WARMUP_ITERATIONS = 5
DEFAULT_ITERATIONS = 20
MIN_ITERATIONS = 1
MAX_ITERATIONS = 100

SHAPE_SETS = {
    "frozen": ((4096, 4096, 4096), (8192, 8192, 8192), (16384, 512, 4096), (32768, 512, 4096),
               (512, 16384, 4096)),
    "c1": ((512, 512, 512),),
    "c4": ((4096, 4096, 4096), (8192, 8192, 8192), (16384, 16384, 16384)),
    "c5": ((8192, 4096, 4096), (8192, 14336, 4096), (8192, 4096, 14336), (8192, 128256, 4096)),
}

CANDIDATES = (
    {"method": "b200", "variant": "persistent_1cta", "mode": "1cta", "mma_tiler": (128, 256),
     "cluster": (1, 1), "use_2cta_instrs": False},
    {"method": "b200", "variant": "persistent_2cta", "mode": "2cta", "mma_tiler": (256, 256),
     "cluster": (2, 1), "use_2cta_instrs": True},
    {"method": "b200", "variant": "persistent_2cta_m512", "mode": "2cta_m512",
     "mma_tiler": (512, 256), "cluster": (2, 1), "use_2cta_instrs": True},
    {"method": "b200", "variant": "persistent_2cta_n128", "mode": "2cta_n128",
     "mma_tiler": (256, 128), "cluster": (2, 1), "use_2cta_instrs": True},
    # The library's own choice per shape (B200_MODE_AUTO).
    {"method": "b200", "variant": "persistent_auto", "mode": "auto", "mma_tiler": None,
     "cluster": None, "use_2cta_instrs": None},
    {"method": "cublas", "variant": "torch_matmul", "mode": None, "mma_tiler": None,
     "cluster": None, "use_2cta_instrs": None},
    # NVIDIA's CuTe DSL Blackwell examples, the reference's three CuTe DSL candidates
    # (gemm_comparison.py:214-265); context baselines, see cutedsl_baseline.py.
    {"method": "cutedsl", "variant": "cutedsl_nonpersistent_1cta", "mode": None,
     "mma_tiler": None, "cluster": None, "use_2cta_instrs": None},
    {"method": "cutedsl", "variant": "cutedsl_persistent_1cta", "mode": None,
     "mma_tiler": None, "cluster": None, "use_2cta_instrs": None},
    {"method": "cutedsl", "variant": "cutedsl_persistent_2cta", "mode": None,
     "mma_tiler": None, "cluster": None, "use_2cta_instrs": None},
    # The reference's own cuBLASLt bridge (cublaslt_bridge_p35.cu), built unmodified by
    # baseline/build_ref_bridge.sh; context baseline for its five frozen shapes, fp32 D.
    {"method": "cublaslt", "variant": "heuristic_first_supported", "mode": None,
     "mma_tiler": None, "cluster": None, "use_2cta_instrs": None},
)
REF_BRIDGE = "baseline/_ref/libcublaslt_bridge_p35.so"
BASELINE_VARIANTS = ("heuristic_first_supported", "torch_matmul")

# Rows carry the reference's 100 p35.v1 columns (src/gemm/gemm_comparison.py:324-440)
# in its order; the default b200 schema appends the B200-specific columns.
P35_FIELDS = row_contracts.P35_FIELDS
B200_EXTRA_FIELDS = ("operands", "stages", "grid_ctas", "schedule", "roofline_fraction",
                     "peak_tflops", "n_gpus")
CSV_FIELDS = P35_FIELDS + B200_EXTRA_FIELDS
KERNEL_SOURCE = "gb300-gemm-anatomy_b200/csrc/gemm_sm100.cu"


class UsageError(Exception):
    pass


def bounded_int(lo, hi):
    def parse(text):
        try:
            v = int(text, 10)
        except ValueError as exc:
            raise argparse.ArgumentTypeError(f"{text!r} is not an integer") from exc
        if v < lo or v > hi:
            raise argparse.ArgumentTypeError(f"{v} is outside [{lo}, {hi}]")
        return v
    return parse


def parse_shape(text: str):
    parts = text.lower().split("x")
    if len(parts) != 3:
        raise argparse.ArgumentTypeError(f"shape {text!r} must be MxNxK")
    try:
        m, n, k = (int(p) for p in parts)
    except ValueError as exc:
        raise argparse.ArgumentTypeError(f"shape {text!r} must be MxNxK integers") from exc
    if min(m, n, k) <= 0:
        raise argparse.ArgumentTypeError(f"shape {text!r} must be positive")
    return (m, n, k)


def build_arg_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="gemm_comparison",
                                description=__doc__.split("\n\n")[0])
    p.add_argument("--warmup-iterations", type=bounded_int(MIN_ITERATIONS, MAX_ITERATIONS),
                   default=DEFAULT_WARMUP_ITERATIONS, metavar="N")
    p.add_argument("--iterations", type=bounded_int(MIN_ITERATIONS, MAX_ITERATIONS),
                   default=DEFAULT_ITERATIONS, metavar="N")
    p.add_argument("--self-test", action="store_true",
                   help="run the GPU-free self-test and exit (no CUDA, nothing on stdout)")
    p.add_argument("--shapes", choices=sorted(SHAPE_SETS), default="frozen")
    p.add_argument("--shape", type=parse_shape, action="append", default=None,
                   help="explicit MxNxK (repeatable); overrides --shapes")
    p.add_argument("--operands", choices=("ref-compat", "config"), default="ref-compat")
    p.add_argument("--out-dtype", choices=("f32", "bf16"), default="f32")
    p.add_argument("--candidates", default="persistent_auto,torch_matmul",
                   help="comma list of persistent_auto, persistent_1cta, persistent_2cta, "
                        "persistent_2cta_m512, persistent_2cta_n128, "
                        "torch_matmul, "
                        "heuristic_first_supported (the reference's cuBLASLt bridge), "
                        "cutedsl_nonpersistent_1cta, cutedsl_persistent_1cta, "
                        "cutedsl_persistent_2cta (NVIDIA's CuTe DSL examples)")
    p.add_argument("--schedule", choices=("auto", "dynamic", "streamk"), default="auto",
                   help="tile schedule of the B200 candidates (auto: the library's choice)")
    p.add_argument("--schema", choices=("b200", "p35"), default="b200",
                   help="p35: exactly the reference's 100 p35.v1 columns; b200: those plus "
                        "the B200 columns (operands, stages, grid, schedule, roofline)")
    p.add_argument("--run-kind", choices=("smoke", "benchmark"), default="smoke")
    p.add_argument("--peak-tflops", type=float, default=None,
                   help="roofline denominator (default: MEASURED_PEAKS.json bf16_tflops)")
    return p


def select_candidates(spec: str):
    names = [s.strip() for s in spec.split(",") if s.strip()]
    known = {c["variant"]: c for c in CANDIDATES}
    bad = [n for n in names if n not in known]
    if bad or not names:
        raise UsageError(f"unknown candidate(s) {bad}; choose from {sorted(known)}")
    return [known[n] for n in names]


def comparison_fields(flop: int, times_ms, variants):
    """tflops, ratio/gap vs the cuBLAS baseline (if present) and rank, per candidate."""
    from ..formulas import compute_ratio_and_gap, compute_tflops
    tflops = [compute_tflops(flop, t) for t in times_ms]
    base_name = next((v for v in BASELINE_VARIANTS if v in variants), None)
    base = tflops[variants.index(base_name)] if base_name else None
    order = sorted(range(len(times_ms)), key=lambda i: (times_ms[i], i))
    rank = [0] * len(times_ms)
    for pos, i in enumerate(order):
        rank[i] = pos + 1
    out = []
    for i, tf in enumerate(tflops):
        if base is None:
            ratio, gap = None, None
        elif variants[i] == base_name:
            ratio, gap = 1.0, 0.0
        else:
            ratio, gap = compute_ratio_and_gap(tf, base)
        out.append({"tflops": tf, "throughput_ratio_vs_cublaslt": ratio,
                    "gap_to_cublaslt_pct": gap, "rank_within_shape": rank[i]})
    return out


def format_csv(rows, fields=CSV_FIELDS) -> str:
    buf = io.StringIO()
    buf.write(",".join(fields) + "\n")
    for r in rows:
        vals = []
        for f in fields:
            v = r.get(f)
            if v is None:
                vals.append("")
            elif isinstance(v, bool):
                vals.append("true" if v else "false")
            elif isinstance(v, float):
                vals.append(repr(v) if math.isfinite(v) else "nan")
            else:
                s = str(v)
                vals.append('"' + s.replace('"', '""') + '"' if ("," in s or '"' in s) else s)
        buf.write(",".join(vals) + "\n")
    return buf.getvalue()


def run_self_test() -> int:
    """GPU-free checks of the argument contract, formulas and CSV emitter."""
    from .. import formulas
    failures = []

    def expect(cond, what):
        if not cond:
            failures.append(what)

    parser = build_arg_parser()
    saved, sys.stderr = sys.stderr, io.StringIO()  # argparse prints usage on rejection
    try:
        _expect_rejections(parser, expect)
    finally:
        sys.stderr = saved
    ns = parser.parse_args([])
    expect(ns.iterations == 20 and ns.warmup_iterations == 5, "defaults")
    _rest_of_self_test(expect, formulas)
    for f in failures:
        print(f"gemm_comparison: SELF_TEST FAIL {f}", file=sys.stderr)
    print(f"gemm_comparison: SELF_TEST_RESULT={'PASS' if not failures else 'FAIL'}",
          file=sys.stderr)
    return 0 if not failures else 1


def _expect_rejections(parser, expect):
    for bad in (["--iterations", "0"], ["--iterations", "101"], ["--warmup-iterations", "x"],
                ["--shape", "1x2"], ["--shape", "0x1x1"]):
        try:
            parser.parse_args(bad)
            expect(False, f"accepted {bad}")
        except SystemExit:
            pass


def _rest_of_self_test(expect, formulas):
    expect(formulas.compute_flop_count(8192, 8192, 8192) == 1099511627776, "flop 8192^3")
    expect(abs(formulas.compute_tflops(1099511627776, 0.519) - 2118.5195140192677) < 1e-9,
           "tflops")
    rows = comparison_fields(2 * 512 ** 3, [0.010, 0.008, 0.020],
                             ["persistent_1cta", "persistent_2cta", "torch_matmul"])
    expect([r["rank_within_shape"] for r in rows] == [2, 1, 3], "ranks")
    expect(rows[2]["throughput_ratio_vs_cublaslt"] == 1.0 and rows[2]["gap_to_cublaslt_pct"] == 0.0,
           "baseline ratio")
    expect(abs(rows[1]["throughput_ratio_vs_cublaslt"] - 2.5) < 1e-12, "ratio")
    expect(abs(rows[1]["gap_to_cublaslt_pct"] + 150.0) < 1e-9, "gap")
    text = format_csv([{"shape_id": "1x2", "method": "a,b", "tflops": 1.5, "publishable": False}])
    lines = text.strip().split("\n")
    expect(len(lines) == 2 and lines[0].split(",") == list(CSV_FIELDS), "csv header")
    expect('"a,b"' in lines[1] and "false" in lines[1], "csv quoting")
    try:
        select_candidates("nope")
        expect(False, "accepted unknown candidate")
    except UsageError:
        pass


def _peak(args):
    if args.peak_tflops:
        return args.peak_tflops
    import json
    from pathlib import Path
    p = Path(__file__).resolve().parents[3] / "MEASURED_PEAKS.json"
    if p.is_file():
        return float(json.loads(p.read_text())["bf16_tflops"])
    return 1590.0


def _ref_plan_info_type():
    """ctypes mirror of the reference bridge's P35PlanInfo: 45 int64 members then three
    doubles, in the order of src/gemm/cublaslt_bridge_p35.cu's struct (read back through
    p35_plan_create's info argument; size checked against p35_plan_info_size)."""
    import ctypes
    ints = ("abi_version", "cublaslt_version", "shape_index", "m", "n", "k", "batch_count",
            "lda", "ldb", "ldc", "ldd", "transa", "transb", "order_a", "order_b", "order_c",
            "order_d", "type_a", "type_b", "type_c", "type_d", "compute_type", "scale_type",
            "pointer_mode", "epilogue", "search_mode", "workspace_limit_bytes",
            "workspace_bytes", "workspace_is_null", "heuristic_requested",
            "heuristic_returned", "heuristic_index", "alignment_a_bytes", "alignment_b_bytes",
            "alignment_c_bytes", "alignment_d_bytes", "algo_id", "tile_id", "stages_id",
            "split_k", "reduction_scheme", "cta_swizzling", "custom_option", "inner_shape_id",
            "cluster_shape_id")

    class RefPlanInfo(ctypes.Structure):
        _fields_ = [(n, ctypes.c_int64) for n in ints] + [
            ("waves_count", ctypes.c_double), ("alpha", ctypes.c_double), ("beta", ctypes.c_double)]
    return RefPlanInfo


class _RefBridgePlan:
    """One plan of the reference's unmodified cuBLASLt bridge (p35_* C ABI)."""

    def __init__(self, m, n, k, a, b, out, stream):
        import ctypes
        from pathlib import Path
        path = Path(__file__).resolve().parents[3] / REF_BRIDGE
        if not path.is_file():
            raise UsageError(f"{path} is missing; build it with baseline/build_ref_bridge.sh")
        lib = ctypes.CDLL(str(path))
        lib.p35_plan_info_size.restype = ctypes.c_size_t
        lib.p35_last_error.restype = ctypes.c_char_p
        lib.p35_plan_create.restype = ctypes.c_int
        lib.p35_plan_create.argtypes = [ctypes.c_int64] * 3 + [ctypes.c_void_p] * 5 + [
            ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
        for name in ("p35_plan_execute", "p35_stream_synchronize", "p35_plan_destroy"):
            getattr(lib, name).restype = ctypes.c_int
            getattr(lib, name).argtypes = [ctypes.c_void_p]
        info_t = _ref_plan_info_type()
        if int(lib.p35_plan_info_size()) != ctypes.sizeof(info_t):
            raise UsageError(f"reference bridge info size {int(lib.p35_plan_info_size())} != "
                             f"mirror {ctypes.sizeof(info_t)}")
        self.info = info_t()
        self.plan = ctypes.c_void_p()
        rc = lib.p35_plan_create(m, n, k, a.data_ptr(), b.data_ptr(), out.data_ptr(),
                                 out.data_ptr(), int(stream.cuda_stream), ctypes.byref(self.plan),
                                 ctypes.byref(self.info))
        if rc != 0:
            raise UsageError(f"reference bridge refused {m}x{n}x{k}: {lib.p35_last_error()!r}")
        self.lib = lib

    def row_fields(self) -> dict:
        """The cuBLASLt columns of a p35 row, as the reference writes them
        (gemm_comparison.py:1578-1614)."""
        i = self.info
        out = dict(row_contracts.CUBLASLT_FROZEN_TEXT)
        for f in ("lda", "ldb", "ldc", "ldd", "workspace_bytes", "alignment_a_bytes",
                  "alignment_b_bytes", "alignment_c_bytes", "alignment_d_bytes",
                  "heuristic_returned", "heuristic_index", "algo_id", "tile_id", "stages_id",
                  "split_k", "reduction_scheme", "cta_swizzling", "custom_option",
                  "inner_shape_id", "cluster_shape_id", "cublaslt_version"):
            out[f] = int(getattr(i, f))
        out["alpha"], out["beta"] = float(i.alpha), float(i.beta)
        out["waves_count"] = float(i.waves_count)
        return out

    def execute(self):
        if self.lib.p35_plan_execute(self.plan) != 0:
            raise RuntimeError(f"p35_plan_execute failed: {self.lib.p35_last_error()!r}")

    def synchronize(self):
        if self.lib.p35_stream_synchronize(self.plan) != 0:
            raise RuntimeError(f"p35_stream_synchronize failed: {self.lib.p35_last_error()!r}")

    def destroy(self):
        if self.plan:
            self.lib.p35_plan_destroy(self.plan)
            self.plan = ctypes_null()


def ctypes_null():
    import ctypes
    return ctypes.c_void_p()


def _factory_sha256(opname: str) -> str:
    """sha256 of the source that produced the operands (the reference records its
    operand factory's source hash, gemm_comparison.py:3098-3125)."""
    import hashlib
    import inspect
    from pathlib import Path
    try:
        if opname.startswith("cutlass"):
            import cutlass.torch
            src = inspect.getsourcefile(cutlass.torch)
        else:
            from .. import operands
            src = inspect.getsourcefile(operands)
        return hashlib.sha256(Path(src).read_bytes()).hexdigest()
    except Exception:  # noqa: BLE001
        return row_contracts.NOT_APPLICABLE


def run_provenance(torch) -> dict:
    """The provenance block of every row (gemm_comparison.py:1178-1230)."""
    from pathlib import Path
    dev = row_contracts.device_provenance(torch, 0)
    kernel = Path(__file__).resolve().parents[3] / KERNEL_SOURCE
    ident = row_contracts.file_identity(kernel) if kernel.is_file() else {"sha256": None, "blob": None}
    return {"gpu_name": dev["gpu_name"], "gpu_uuid": dev["gpu_uuid"],
            "compute_capability": dev["compute_capability"],
            "driver_version": dev["driver_version"],
            "cuda_toolkit_version": row_contracts.cuda_toolkit_version(),
            "torch_cuda_version": dev["torch_cuda_version"],
            "cutedsl_version": row_contracts.cutedsl_version(),
            "kernel_sha256": ident["sha256"], "kernel_blob": ident["blob"],
            **row_contracts.git_state()}


def execute_measurement(args) -> str:
    import time

    import torch

    from .. import check, operands
    from ..gemm import GemmPlan

    if not torch.cuda.is_available():
        raise RuntimeError("no CUDA device is visible")
    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device("cuda", 0)
    shapes = args.shape if args.shape else SHAPE_SETS[args.shapes]
    cands = select_candidates(args.candidates)
    out_dtype = torch.float32 if args.out_dtype == "f32" else torch.bfloat16
    peak = _peak(args)
    prov = run_provenance(torch)
    rows = []
    stream = torch.cuda.current_stream(dev)
    for si, (m, n, k) in enumerate(shapes):
        if args.operands == "ref-compat":
            if operands.ref_compat_available():
                a_h, b_h = operands.ref_compat_operands(m, n, k)
                seed, opname = operands.REF_SEED, "cutlass.torch.matrix(seed 1111)"
            else:
                a_h, b_h = operands.integer_operands(m, n, k)
                seed, opname = operands.REF_SEED, "integer{-2..1}(seed 1111)"
        else:
            a_h, b_h = operands.uniform_operands(m, n, k, seed=0) if (m, n, k) == (512, 512, 512) \
                else operands.normal_operands(m, n, k, seed=1, std_a=0.1, std_b=0.1)
            seed, opname = (0 if (m, n, k) == (512, 512, 512) else 1), "config"
        a = a_h.to(dev)
        b = b_h.to(dev)
        # The reference's oracle: IEEE fp32 matmul on the GPU (gemm_comparison.py:2705-2722).
        torch.backends.cuda.matmul.fp32_precision = "ieee"
        reference = torch.einsum("mk,nk->mn", a.float(), b.float())
        out = torch.empty((m, n), dtype=out_dtype, device=dev)
        times, metas = [], []
        for cand in cands:
            out.fill_(float("nan"))
            torch.cuda.synchronize()
            t_setup = time.perf_counter()
            extra = {}
            if cand["method"] == "b200":
                plan = GemmPlan(a, b, out, mode=cand["mode"], stream=stream)
                launch = plan.execute
                meta = plan.info
                extra["schedule"] = plan.schedule
            elif cand["method"] == "cublaslt":
                if out_dtype != torch.float32:
                    raise UsageError("the reference cuBLASLt bridge writes fp32 D only")
                plan = _RefBridgePlan(m, n, k, a, b, out, stream)
                launch = plan.execute
                meta = {}
                extra.update(plan.row_fields())
            elif cand["method"] == "cutedsl":
                from . import cutedsl_baseline
                ok, why = cutedsl_baseline.available()
                if not ok:
                    raise UsageError(f"{cand['variant']} is unavailable on this box: {why}")
                plan = cutedsl_baseline.CuteDslPlan(cand["variant"], a, b, out, stream)
                launch = plan.execute
                meta = {}
                ident = row_contracts.file_identity(plan.source)
                extra.update(plan.meta)
                extra.update({"upstream_kernel_git_blob": ident["blob"],
                              "upstream_kernel_sha256": ident["sha256"]})
            else:
                plan = None

                def launch(o=out):
                    # bf16 x bf16 with fp32 accumulation; fp32 D via aten::mm.dtype.
                    if o.dtype == torch.bfloat16:
                        torch.matmul(a, b.T, out=o)
                    else:
                        torch.mm(a, b.T, out_dtype=torch.float32, out=o)
                meta = {}
            setup_ms = (time.perf_counter() - t_setup) * 1e3 \
                if plan is not None and cand["method"] != "cutedsl" else None
            f0 = torch.cuda.Event(enable_timing=True)
            f1 = torch.cuda.Event(enable_timing=True)
            f0.record(stream)
            launch()
            f1.record(stream)
            if plan is not None:
                plan.synchronize()
            torch.cuda.synchronize()
            first_ms = f0.elapsed_time(f1)
            label = f"{m}x{n}x{k}/{cand['variant']}"
            if out_dtype == torch.float32:
                max_abs, max_rel = check.validate_result(label, reference, out)
            else:
                stats = check.bf16_tolerance_check(label, reference, out, k,
                                                   float(a_h.float().abs().max()),
                                                   float(b_h.float().abs().max()))
                max_abs, max_rel = stats["max_abs_error"], stats["rel_fro"]
            for _ in range(args.warmup_iterations):
                launch()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.iterations):
                launch()
            e1.record(stream)
            torch.cuda.synchronize()
            if plan is not None:
                plan.synchronize()
                plan.destroy()
            times.append(e0.elapsed_time(e1) / args.iterations)
            metas.append((cand, meta, max_abs, max_rel, setup_ms, first_ms, extra))
        flop = 2 * m * n * k
        comp = comparison_fields(flop, times, [c["variant"] for c in cands])
        # The best of the CuTe DSL rows when there are any (the reference's meaning),
        # else the best of the B200 kernel's rows.
        own = [i for i, c in enumerate(cands) if c["method"] == "cutedsl"] or \
            [i for i, c in enumerate(cands) if c["method"] == "b200"]
        best_own = cands[min(own, key=lambda i: (times[i], i))]["variant"] if own else None
        for ci, ((cand, meta, max_abs, max_rel, setup_ms, first_ms, extra), t, cf) in enumerate(
                zip(metas, times, comp)):
            own_kernel = cand["method"] == "b200"
            cta = meta.get("cta_group") or 1
            row = {
                "schema_version": SCHEMA_VERSION, "experiment": EXPERIMENT, "unit": UNIT,
                "run_kind": args.run_kind,
                "shape_index": si, "shape_id": f"{m}x{n}x{k}x1", "candidate_index": ci,
                "method": cand["method"], "variant": cand["variant"], "m": m, "n": n, "k": k,
                "l": 1, "ab_dtype": "BFloat16", "acc_dtype": "Float32",
                "c_dtype": "Float32" if out_dtype == torch.float32 else "BFloat16",
                "a_major": "k", "b_major": "k", "c_major": "n",
                "seed": seed, "operands": opname,
                "reference": "torch_fp32_ieee_einsum", "atol": check.REF_ATOL,
                "rtol": check.REF_RTOL, "correctness": "PASS", "max_abs_error": max_abs,
                "max_rel_error": max_rel, "setup_time_ms": setup_ms, "first_launch_ms": first_ms,
                "kernel_time_ms": t, "cache_mode": "hot",
                "warmup_iterations": args.warmup_iterations, "iterations": args.iterations,
                "flop_count": flop, "best_cutedsl_variant": best_own,
                "is_best_cutedsl": cand["variant"] == best_own,
                "roofline_fraction": cf["tflops"] / peak,
                "peak_tflops": peak, "n_gpus": 1, "gpu_name": prov["gpu_name"],
                "gpu_uuid": prov["gpu_uuid"], "compute_capability": prov["compute_capability"],
                "driver_version": prov["driver_version"],
                "cuda_toolkit_version": prov["cuda_toolkit_version"],
                "torch_cuda_version": prov["torch_cuda_version"],
                "cutedsl_version": prov["cutedsl_version"],
                "operand_factory_sha256": _factory_sha256(opname),
                "git_commit": prov["git_commit"], "git_dirty": prov["git_dirty"],
                "publishable": False,
                **cf, **extra,
            }
            if own_kernel:
                row.update({
                    "scheduler": f"{extra['schedule']}_persistent",
                    "mma_tiler_m": meta.get("tile_m"), "mma_tiler_n": meta.get("tile_n"),
                    "cluster_m": cta, "cluster_n": 1, "use_2cta_instrs": cta == 2,
                    "use_tma_store": True,
                    "max_active_clusters": (meta.get("grid_ctas") or 0) // cta,
                    "upstream_kernel_file": KERNEL_SOURCE,
                    "upstream_kernel_git_blob": prov["kernel_blob"],
                    "upstream_kernel_sha256": prov["kernel_sha256"],
                    "stages": meta.get("stages"), "grid_ctas": meta.get("grid_ctas"),
                    "waves_count": meta.get("waves"),
                })
            rows.append(row)
            print(f"gemm_comparison: {m}x{n}x{k} {cand['variant']}: {t:.4f} ms "
                  f"{cf['tflops']:.1f} TFLOP/s max_abs={max_abs:.3g}", file=sys.stderr)
        del a, b, out, reference
        torch.cuda.empty_cache()
    if args.schema == "p35":
        return format_csv([row_contracts.p35_text(r) for r in rows], P35_FIELDS)
    return format_csv([{**r, **row_contracts.p35_text(r)} for r in rows], CSV_FIELDS)


def main(argv=None) -> int:
    parser = build_arg_parser()
    try:
        args = parser.parse_args(argv)
    except SystemExit as exc:
        return 2 if exc.code else 0
    if args.self_test:
        return run_self_test()
    if args.schedule != "auto":
        import os
        os.environ["B200_GEMM_SCHEDULE"] = args.schedule  # read at plan creation
    try:
        select_candidates(args.candidates)
        text = execute_measurement(args)
    except UsageError as exc:
        print(f"gemm_comparison: ERROR: {exc}", file=sys.stderr)
        return 2
    except Exception as exc:  # every failure: no CSV, exit 1
        print(f"gemm_comparison: ERROR: {type(exc).__name__}: {exc}", file=sys.stderr)
        return 1
    sys.stdout.write(text)
    sys.stdout.flush()
    return 0


if __name__ == "__main__":
    sys.exit(main())
