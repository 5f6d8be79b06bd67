"""UMMA throughput driver: tcgen05.mma kind::f16 with operands resident in SMEM.

Mirrors the reference's umma_1sm / umma_2sm binaries (src/compute/umma_1sm.cu
main :1120, run_once :1020-1060): validate the known answer exactly first,
then warm up and time `repetitions` launches of `iterations` commit rounds,
reporting FLOP/cycle/SM from the leader's %clock64 (umma_1sm.cu:990-991) and
TFLOP/s from CUDA events. --self-test validates every (mode, N, depth).
Additions: depth in {4,16,32,64,128,256} (the union of the reference grid and
the benchmark config), --num-ctas (run the probe on every SM at once), and
--operands uniform (seeded uniform[-1,1) bf16, checked with a tolerance).
"""
from __future__ import annotations

import argparse
import datetime
import sys

from . import row_contracts

# The reference binaries' 37 columns (src/compute/umma_1sm.cu:976-983, the same in
# umma_2sm.cu) in their order; the default b200 schema appends the B200 columns.
REF_FIELDS = row_contracts.UMMA_FIELDS
B200_EXTRA_FIELDS = (
    "schema_version_b200", "num_ctas", "operands", "leader_cycles", "flop_per_launch",
    "flops_per_cycle_per_sm", "kernel_time_ms", "tflops", "tflops_per_sm", "sm_count",
)
CSV_FIELDS = REF_FIELDS + B200_EXTRA_FIELDS


def build_arg_parser():
    p = argparse.ArgumentParser(prog="umma", description=__doc__.split("\n\n")[0])
    p.add_argument("--self-test", action="store_true")
    p.add_argument("--mode", choices=("1sm", "2sm"), default="1sm")
    p.add_argument("--n", type=int, choices=(64, 128, 256), default=256)
    p.add_argument("--depth", type=int, choices=(4, 16, 32, 64, 128, 256), default=256)
    p.add_argument("--iterations", type=int, default=1000)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--repetitions", type=int, default=30)
    p.add_argument("--num-ctas", default="1", help="'1', 'all' (one CTA per SM) or a count")
    p.add_argument("--operands", choices=("pattern", "uniform"), default="pattern")
    p.add_argument("--sweep", action="store_true", help="all (mode, N, depth) combinations")
    p.add_argument("--run-kind", choices=("smoke", "benchmark"), default="benchmark")
    p.add_argument("--schema", choices=("b200", "ref"), default="b200",
                   help="ref: exactly the reference binaries' 37 columns")
    return p


def _identity():
    """gpu_uuid, CUDA driver / runtime versions and git state (reference provenance)."""
    import torch

    from .. import _lib
    info = _lib.device_probe(0)
    return {"gpu_uuid": f"GPU-{torch.cuda.get_device_properties(0).uuid}",
            "compute_capability": f"{info['cc_major']}.{info['cc_minor']}",
            "cuda_driver_version": info["driver_version"],
            "cuda_runtime_version": info["runtime_version"], **row_contracts.git_state()}


def run_case(cta_group, n, depth, args, num_ctas, sms, name):
    import numpy as np
    import torch

    from .. import formulas
    from ..umma import run_probe

    a = b = None
    m = 128 * cta_group
    if args.operands == "uniform":
        g = torch.Generator().manual_seed(0)
        a = (torch.rand((m, 16), generator=g) * 2 - 1).to(torch.bfloat16)
        b = (torch.rand((n, 16), generator=g) * 2 - 1).to(torch.bfloat16)
    d, cycles, status = run_probe(cta_group, n, depth, iterations=2, a=a, b=b)
    torch.cuda.synchronize()
    if int(status.item()) != 0:
        raise RuntimeError(f"probe status {int(status.item()):#x}")
    if a is None:
        r = np.arange(m)[:, None]
        kk = np.arange(16)[None, :]
        A = ((r + 3 * kk) % 7) - 3
        c = np.arange(n)[None, :]
        kc = np.arange(16)[:, None]
        B = ((2 * kc + c) % 5) - 2
        want = depth * (A @ B).astype(np.float64)
        max_err = float(np.abs(d.cpu().double().numpy() - want).max())
        ok = max_err == 0.0
    else:
        want = depth * (a.double() @ b.double().T).numpy()
        max_err = float(np.abs(d.cpu().double().numpy() - want).max())
        ok = max_err <= depth * 16 * 2 ** -22 * (1 + np.abs(want).max())
    if not ok:
        raise RuntimeError(f"UMMA {name} N={n} depth={depth}: D mismatch")
    rows = []
    if args.self_test:
        return rows
    for _ in range(args.warmup):
        run_probe(cta_group, n, depth, iterations=args.iterations, a=a, b=b, num_ctas=num_ctas)
    torch.cuda.synchronize()
    flop = formulas.umma_flop_count(m, n, depth, args.iterations)
    ctas = max(num_ctas, 1)
    for rep in range(args.repetitions):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        _, cyc, st = run_probe(cta_group, n, depth, iterations=args.iterations, timed=True,
                               a=a, b=b, num_ctas=num_ctas)
        e1.record()
        torch.cuda.synchronize()
        if int(st.item()) != 0:
            raise RuntimeError(f"probe status {int(st.item()):#x}")
        ms = e0.elapsed_time(e1)
        leader = int(cyc[0].item())
        total_flop = flop * ctas
        total_umma = depth * args.iterations
        rows.append({
            "schema_version": "1", "schema_version_b200": "b200.umma.1",
            "timestamp_utc": datetime.datetime.now(datetime.timezone.utc).strftime(
                "%Y-%m-%dT%H:%M:%SZ"),
            "run_kind": getattr(args, "run_kind", "benchmark"), "publishable": "false",
            "warmup_iterations": args.warmup, "repetitions": args.repetitions,
            "umma_per_iteration": depth, "total_umma": total_umma,
            "flops_per_umma": 2 * m * n * 16, "total_flops": flop, "elapsed_cycles": leader,
            "cycles_per_umma": f"{leader / total_umma:.6f}",
            "flops_per_cycle": f"{flop / leader:.6f}" if leader else "0.000000",
            "threads_per_cta": 128, "grid_blocks": ctas * cta_group, "tmem_columns": n,
            "operand_path": "smem_smem", "input_type": "bf16", "accumulator_type": "fp32",
            "mismatches": 0, "max_abs_error": f"{max_err:.6f}", **_identity(),
            "method": name, "cta_group": cta_group, "m": m,
            "n": n, "k": 16, "depth": depth, "iterations": args.iterations, "num_ctas": ctas,
            "sample_index": rep, "operands": args.operands, "correctness": "OK",
            "leader_cycles": leader, "flop_per_launch": total_flop,
            "flops_per_cycle_per_sm": formulas.flops_per_cycle_per_sm(flop, leader, cta_group),
            "kernel_time_ms": ms, "tflops": total_flop / ms / 1e9,
            "tflops_per_sm": total_flop / ms / 1e9 / (ctas * cta_group), "sm_count": sms,
            "gpu_name": torch.cuda.get_device_properties(0).name,
        })
    return rows


def main(argv=None) -> int:
    parser = build_arg_parser()
    try:
        args = parser.parse_args(argv)
    except SystemExit as exc:
        return 2 if exc.code else 0
    if args.iterations < 1 or args.repetitions < 1 or args.warmup < 0:
        print("umma: ERROR: --iterations/--repetitions must be >= 1", file=sys.stderr)
        return 2
    try:
        import torch
        if not torch.cuda.is_available():
            raise RuntimeError("no CUDA device is visible")
        sms = torch.cuda.get_device_properties(0).multi_processor_count
        if args.self_test or args.sweep:
            cases = [(g, n, d) for g in (1, 2) for n in (64, 128, 256)
                     for d in (4, 16, 32, 64, 128, 256)]
        else:
            cases = [(1 if args.mode == "1sm" else 2, args.n, args.depth)]
        rows = []
        for (g, n, d) in cases:
            if args.num_ctas == "all":
                num = sms // g
            else:
                num = int(args.num_ctas)
            name = "umma_1sm" if g == 1 else "umma_2sm"
            rows += run_case(g, n, d, args, num, sms, name)
            if args.self_test:
                print(f"umma: SELF_TEST {name} N={n} depth={d} PASS", file=sys.stderr)
        if args.self_test:
            print("umma: SELF_TEST_RESULT=PASS", file=sys.stderr)
            return 0
    except Exception as exc:
        print(f"umma: ERROR: {type(exc).__name__}: {exc}", file=sys.stderr)
        return 1
    fields = REF_FIELDS if args.schema == "ref" else CSV_FIELDS
    out = [",".join(fields)]
    for r in rows:
        out.append(",".join(f'"{r[f]}"' if "," in str(r[f]) else str(r[f]) for f in fields))
    sys.stdout.write("\n".join(out) + "\n")
    return 0


if __name__ == "__main__":
    sys.exit(main())
