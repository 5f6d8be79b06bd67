"""Memory-path driver: LDGSTS / TMA global->SMEM streaming, validated then timed.

Mirrors the reference binaries' command line (src/memory/ldgsts.cu:600-710,
src/memory/tma.cu main): --stages {2,4,8}, --bytes-in-flight-kib {16,32,64}
(stage = bytes in flight / stages), --working-set-mib (default 4 x L2, rounded
to whole stages), --passes, --warmup-ms, --repetitions, --run-kind
{smoke,benchmark} (benchmark requires a working set > 2 x L2), --self-test
(validate every specialisation), exit 0/1/2, CSV rows on stdout only after
correctness passed. Additions: --method {ldgsts,tma,tma_sw128},
--ctas-per-sm {1,2,4}, --stage-kib (overrides the bytes-in-flight split),
--fill {pattern,uniform} (SplitMix64 index pattern validated per vector, or a
seeded uniform bf16 buffer whose streamed checksum must equal the host
checksum bit for bit), and --sweep {reference,baseline}.
"""
from __future__ import annotations

import argparse
import sys
import time

from .._lib import ERR_UNSUPPORTED, BridgeError

from . import row_contracts

SCHEMA_VERSION = "b200.mem.1"
# The reference binaries' 37 columns (src/memory/ldgsts.cu:741-752, tma.cu:1028-1039)
# in their order; the default b200 schema appends the roofline and checksum columns.
REF_FIELDS = row_contracts.MEM_FIELDS
B200_EXTRA_FIELDS = ("roofline_fraction", "hbm_peak_gbps", "fill", "checksum_xor", "checksum_sum",
                     "host_checksum_xor", "host_checksum_sum")
CSV_FIELDS = REF_FIELDS + B200_EXTRA_FIELDS


def build_arg_parser():
    p = argparse.ArgumentParser(prog="memory_paths", description=__doc__.split("\n\n")[0])
    p.add_argument("--self-test", action="store_true")
    p.add_argument("--method", choices=("ldgsts", "tma", "tma_sw128"), default="ldgsts")
    p.add_argument("--stages", type=int, choices=(2, 4, 8))
    p.add_argument("--bytes-in-flight-kib", type=int, choices=(16, 32, 64))
    p.add_argument("--stage-kib", type=int, choices=(2, 4, 8, 16, 32, 64))
    p.add_argument("--ctas-per-sm", type=int, choices=(1, 2, 4), default=1)
    p.add_argument("--working-set-mib", type=int)
    p.add_argument("--passes", type=int, default=1)
    p.add_argument("--warmup-ms", type=int, default=100)
    p.add_argument("--repetitions", type=int, default=5)
    p.add_argument("--run-kind", choices=("smoke", "benchmark"))
    p.add_argument("--fill", choices=("pattern", "uniform"), default="pattern")
    p.add_argument("--sweep", choices=("reference", "baseline"))
    p.add_argument("--hbm-peak-gbps", type=float)
    p.add_argument("--schema", choices=("b200", "ref"), default="b200",
                   help="ref: exactly the reference binaries' 37 columns")
    return p


def validate_args(args):
    """Returns an error string or None (the reference's parse_cli rules, ldgsts.cu:692-710)."""
    if args.self_test:
        return None
    if args.sweep:
        if args.run_kind is None:
            return "--run-kind is required"
        return None
    if args.stages is None:
        return "--stages is required (unless --self-test or --sweep)"
    if args.bytes_in_flight_kib is None and args.stage_kib is None:
        return "--bytes-in-flight-kib or --stage-kib is required"
    if args.run_kind is None:
        return "--run-kind is required (unless --self-test)"
    if not 1 <= args.passes <= 1000000:
        return "--passes must be in [1, 1000000]"
    if not 1 <= args.repetitions <= 1000000:
        return "--repetitions must be in [1, 1000000]"
    if args.working_set_mib is not None and not 1 <= args.working_set_mib <= (1 << 20):
        return "--working-set-mib must be in [1, 1048576]"
    return None


def stage_bytes_of(args, stages):
    if args.stage_kib:
        return args.stage_kib * 1024
    return args.bytes_in_flight_kib * 1024 // stages


def reference_grid():
    return [(m, s, bif * 1024 // s, 1) for m in ("ldgsts", "tma") for s in (2, 4, 8)
            for bif in (16, 32, 64)]


def baseline_grid():
    # 16 KiB stages (TMA box 64 x 128 bf16 = 128 x 64 bf16 tile bytes), CTAs/SM x stages.
    return [(m, s, 16384, c) for m in ("ldgsts", "tma_sw128") for c in (1, 2, 4)
            for s in (2, 4, 8)]


def _peak(args):
    if args.hbm_peak_gbps:
        return args.hbm_peak_gbps
    import json
    from pathlib import Path
    p = Path(__file__).resolve().parents[3] / "MEASURED_PEAKS.json"
    if p.is_file():
        return float(json.loads(p.read_text())["hbm_gbs"])
    return 6650.0


def make_buffer(nbytes, fill, dev):
    import torch
    from ..memory_paths import fill_pattern
    if fill == "pattern":
        buf = torch.empty(nbytes // 2, dtype=torch.int16, device=dev)
        fill_pattern(buf)
    else:
        g = torch.Generator(device=dev).manual_seed(2)
        buf = (torch.rand(nbytes // 2, generator=g, device=dev) * 2 - 1).to(torch.bfloat16)
    torch.cuda.synchronize()
    return buf


_HOST_CHECKSUMS = {}


def host_checksum(buf):
    """XOR/sum of the buffer's 32-bit words, computed on the host (cached per buffer)."""
    import numpy as np
    key = (buf.data_ptr(), buf.numel() * buf.element_size())
    if key in _HOST_CHECKSUMS:
        return _HOST_CHECKSUMS[key]
    words = buf.view(__import__("torch").int32).cpu().numpy().view(np.uint32)
    x = int(np.bitwise_xor.reduce(words)) if words.size else 0
    s = int(words.sum(dtype=np.uint64)) & ((1 << 64) - 1)
    _HOST_CHECKSUMS[key] = (x, s)
    return x, s


def run_one(buf, method, stages, stage_bytes, ctas, args, requested, peak, sample_base=0):
    import datetime

    import torch

    from ..memory_paths import StreamPlan

    dev = buf.device
    props = torch.cuda.get_device_properties(dev)
    ident = _identity(dev.index or 0)
    nbytes = buf.numel() * buf.element_size()
    ws = (nbytes // stage_bytes) * stage_bytes
    view = buf.view(torch.uint8)[:ws]
    plan = StreamPlan(view, method, stages, stage_bytes, ctas_per_sm=ctas, passes=args.passes)
    rows = []
    try:
        mode = "validate" if args.fill == "pattern" else "checksum"
        plan.execute(mode)
        r = plan.result()
        hx = hs = None
        if args.fill == "pattern":
            ok = r["mismatches"] == 0
        else:
            hx, hs = host_checksum(view)
            ok = (r["checksum_xor"], r["checksum_sum"]) == (hx, hs)
        if not ok:
            raise RuntimeError(f"{method} stages={stages} stage_bytes={stage_bytes} ctas={ctas}: "
                               f"correctness FAILED ({r})")
        t_end = time.perf_counter() + args.warmup_ms / 1e3
        while time.perf_counter() < t_end:
            plan.execute("sink")
            torch.cuda.synchronize()
        for rep in range(args.repetitions):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            plan.execute("sink")
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            useful = ws * args.passes
            gbps = useful / (ms / 1e3) / 1e9
            rows.append({
                "schema_version": SCHEMA_VERSION,
                "timestamp_utc": datetime.datetime.now(datetime.timezone.utc).strftime(
                    "%Y-%m-%dT%H:%M:%SZ"),
                "run_kind": args.run_kind or "self_test", "method": method,
                "sample_index": sample_base + rep, "stages": stages,
                "tile_width_elements": 64 if method == "tma_sw128" else 128,
                "tile_width_bytes": 128 if method == "tma_sw128" else 256,
                "copies_per_thread_per_stage": stage_bytes // (128 * 16),
                "tile_height": stage_bytes // (128 if method == "tma_sw128" else 256),
                "stage_bytes": stage_bytes, "bytes_in_flight_per_sm": stages * stage_bytes * ctas,
                "vector_bytes": 16, "threads_per_cta": 128, "target_ctas_per_sm": ctas,
                "occupancy_ctas_per_sm": plan.info["occupancy_ctas_per_sm"],
                "grid_blocks": plan.info["grid_ctas"], "sm_count": props.multi_processor_count,
                "smem_reservation_bytes": plan.info["smem_bytes"], "l2_bytes": props.L2_cache_size,
                "requested_working_set_bytes": requested, "working_set_bytes": ws,
                "working_set_l2_ratio": ws / props.L2_cache_size, "passes": args.passes,
                "useful_bytes": useful, "warmup_ms": args.warmup_ms, "kernel_time_ms": ms,
                "effective_gbps": gbps, "roofline_fraction": gbps / peak, "hbm_peak_gbps": peak,
                "correctness": "OK", "mismatches": r["mismatches"], "fill": args.fill,
                "checksum_xor": r["checksum_xor"] if args.fill == "uniform" else None,
                "checksum_sum": r["checksum_sum"] if args.fill == "uniform" else None,
                "host_checksum_xor": hx, "host_checksum_sum": hs, "gpu_name": props.name,
                "compute_capability": f"{props.major}.{props.minor}", **ident,
            })
    finally:
        plan.destroy()
    return rows


_IDENTITY = {}


def _identity(index):
    """gpu_uuid, CUDA driver / runtime versions (cudaDriverGetVersion-style integers)
    and this repository's git state: the reference row's provenance columns."""
    if index not in _IDENTITY:
        import torch

        from .. import _lib
        info = _lib.device_probe(index)
        _IDENTITY[index] = {"gpu_uuid": f"GPU-{torch.cuda.get_device_properties(index).uuid}",
                            "cuda_driver_version": info["driver_version"],
                            "cuda_runtime_version": info["runtime_version"],
                            **row_contracts.git_state()}
    return _IDENTITY[index]


def format_csv(rows, fields=CSV_FIELDS):
    out = [",".join(fields)]
    for r in rows:
        out.append(",".join("" if r.get(f) is None else
                            (f'"{r[f]}"' if "," in str(r[f]) else str(r[f])) for f in fields))
    return "\n".join(out) + "\n"


def main(argv=None) -> int:
    parser = build_arg_parser()
    try:
        args = parser.parse_args(argv)
    except SystemExit as exc:
        return 2 if exc.code else 0
    err = validate_args(args)
    if err:
        print(f"memory_paths: ERROR: {err}", file=sys.stderr)
        return 2
    try:
        import torch
        if not torch.cuda.is_available():
            raise RuntimeError("no CUDA device is visible")
        dev = torch.device("cuda", 0)
        props = torch.cuda.get_device_properties(dev)
        peak = _peak(args)
        if args.self_test:
            # 8 x (SMs x 32 KiB), like the reference self-test (ldgsts.cu:75,474-478).
            nbytes = 8 * props.multi_processor_count * 32 * 1024
            args.fill, args.repetitions, args.warmup_ms = "pattern", 1, 0
            buf = make_buffer(nbytes, "pattern", dev)
            for (m, s, sb, c) in reference_grid() + baseline_grid():
                try:
                    run_one(buf, m, s, sb, c, args, nbytes, peak)
                except BridgeError as exc:
                    if exc.code != ERR_UNSUPPORTED:
                        raise
                    print(f"memory_paths: SELF_TEST {m} stages={s} stage_bytes={sb} ctas={c} "
                          "SKIP (does not fit)", file=sys.stderr)
                    continue
                print(f"memory_paths: SELF_TEST {m} stages={s} stage_bytes={sb} ctas={c} PASS",
                      file=sys.stderr)
            print("memory_paths: SELF_TEST_RESULT=PASS", file=sys.stderr)
            return 0
        requested = (args.working_set_mib * (1 << 20)) if args.working_set_mib \
            else 4 * props.L2_cache_size
        if args.run_kind == "benchmark" and requested <= 2 * props.L2_cache_size:
            raise ValueError(f"working set {requested} is not > 2 x L2; raise --working-set-mib")
        buf = make_buffer(requested - requested % 65536, args.fill, dev)
        if args.sweep:
            grid = reference_grid() if args.sweep == "reference" else baseline_grid()
        else:
            grid = [(args.method, args.stages, stage_bytes_of(args, args.stages), args.ctas_per_sm)]
        rows = []
        for (m, s, sb, c) in grid:
            try:
                rows += run_one(buf, m, s, sb, c, args, requested, peak, sample_base=0)
            except BridgeError as exc:
                if exc.code != ERR_UNSUPPORTED:
                    raise
                print(f"memory_paths: skip {m} stages={s} stage_bytes={sb} ctas={c}: {exc}",
                      file=sys.stderr)
                continue
            best = max(r["effective_gbps"] for r in rows[-args.repetitions:])
            print(f"memory_paths: {m} stages={s} stage_bytes={sb} ctas={c}: {best:.1f} GB/s",
                  file=sys.stderr)
    except Exception as exc:
        print(f"memory_paths: ERROR: {type(exc).__name__}: {exc}", file=sys.stderr)
        return 1
    sys.stdout.write(format_csv(rows, REF_FIELDS if args.schema == "ref" else CSV_FIELDS))
    return 0


if __name__ == "__main__":
    sys.exit(main())
