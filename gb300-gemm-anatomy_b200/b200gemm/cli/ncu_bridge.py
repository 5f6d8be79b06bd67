"""ncu evidence bridge: run one kernel of a command under Nsight Compute and classify it.

Mirrors the reference's p14/p24 ncu bridges (scripts/p14_ncu_bridge.py:85-91,
scripts/p24_ncu_bridge.py:71-81): `--clock-control none`, an exact kernel-name
filter, `--launch-skip` past the validation launches, `--launch-count 1`, a
fixed metric list, CSV parsed here. Two kinds:

  memory  dram__bytes_read.sum / useful bytes -> HBM_VALIDATED / INCONCLUSIVE
          (+READ_AMPLIFICATION), the reference's rule
          (scripts/analyze_exp01_memory_paths_p14.py:1887-1903)
  tensor  sm__pipe_tensor_cycles_active, sm__cycles_elapsed.avg.per_second
          (the SM clock the reference converts FLOP/cycle with,
          scripts/analyze_exp02_umma_throughput_p24.py:114-138) and, given
          --flop, achieved TFLOP/s

Only ever run it on one GPU, after the same command exited 0 without ncu.
Usage:
  python -m b200gemm.cli.ncu_bridge --kind memory --kernel ldgsts_stream \\
      --useful-bytes 1073741824 --skip 1 -- python -m b200gemm.cli.memory_paths ...
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import shutil
import subprocess
import sys

from ..formulas import classify_hbm

METRICS = {
    "memory": ("dram__bytes_read.sum", "dram__bytes_write.sum", "gpu__time_duration.sum",
               "dram__throughput.avg.pct_of_peak_sustained_elapsed"),
    "tensor": ("gpu__time_duration.sum", "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
               "sm__cycles_elapsed.avg.per_second", "dram__bytes_read.sum",
               "sm__inst_executed_pipe_tensor.sum"),
}

UNIT_SCALE = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "ns": 1e-9, "us": 1e-6,
              "usecond": 1e-6, "ms": 1e-3, "msecond": 1e-3, "nsecond": 1e-9, "s": 1.0, "second": 1.0,
              "hz": 1, "Khz": 1e3, "Mhz": 1e6, "Ghz": 1e9, "%": 1, "inst": 1, "": 1}


def ncu_command(kind, kernel, skip, cmd):
    return ["ncu", "--clock-control", "none", "--kernel-name-base", "function", "-k",
            f"regex:{kernel}", "--launch-skip", str(skip), "--launch-count", "1", "--metrics",
            ",".join(METRICS[kind]), "--csv"] + list(cmd)


def parse_csv(text: str) -> dict:
    """{metric: value in base units} of the first profiled launch in ncu --csv output."""
    lines = [ln for ln in text.splitlines() if ln.startswith('"')]
    rows = list(csv.reader(io.StringIO("\n".join(lines))))
    if not rows:
        raise ValueError("no CSV rows in the ncu output")
    h = rows[0]
    mi, ui, vi = h.index("Metric Name"), h.index("Metric Unit"), h.index("Metric Value")
    out = {}
    for r in rows[1:]:
        try:
            v = float(r[vi].replace(",", ""))
        except ValueError:
            continue
        out.setdefault(r[mi], v * UNIT_SCALE.get(r[ui], 1))
    return out


def summarise(kind, metrics, useful_bytes=None, flop=None):
    res = {"kind": kind, "metrics": metrics}
    if kind == "memory":
        cls, flags, ratio = classify_hbm(metrics.get("dram__bytes_read.sum"), float(useful_bytes))
        res.update(classification=cls, flags=flags, dram_read_ratio=ratio)
        t = metrics.get("gpu__time_duration.sum")
        if t:
            res["effective_gbps"] = float(useful_bytes) / t / 1e9
    else:
        t = metrics.get("gpu__time_duration.sum")
        if flop and t:
            res["tflops"] = flop / t / 1e12
        res["sm_clock_ghz"] = metrics.get("sm__cycles_elapsed.avg.per_second", 0) / 1e9
    return res


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if "--" not in argv:
        print("ncu_bridge: ERROR: give the command after --", file=sys.stderr)
        return 2
    i = argv.index("--")
    ap = argparse.ArgumentParser(prog="ncu_bridge")
    ap.add_argument("--kind", choices=sorted(METRICS), required=True)
    ap.add_argument("--kernel", required=True)
    ap.add_argument("--skip", type=int, default=1)
    ap.add_argument("--useful-bytes", type=int)
    ap.add_argument("--flop", type=float)
    try:
        args = ap.parse_args(argv[:i])
    except SystemExit as exc:
        return 2 if exc.code else 0
    if args.kind == "memory" and not args.useful_bytes:
        print("ncu_bridge: ERROR: --useful-bytes is required for --kind memory", file=sys.stderr)
        return 2
    if shutil.which("ncu") is None:
        print("ncu_bridge: ERROR: ncu not found", file=sys.stderr)
        return 1
    proc = subprocess.run(ncu_command(args.kind, args.kernel, args.skip, argv[i + 1:]),
                          capture_output=True, text=True)
    if proc.returncode != 0:
        print(proc.stderr[-2000:], file=sys.stderr)
        return 1
    try:
        res = summarise(args.kind, parse_csv(proc.stdout), args.useful_bytes, args.flop)
    except ValueError as exc:
        print(f"ncu_bridge: ERROR: {exc}", file=sys.stderr)
        return 1
    print(json.dumps(res))
    return 0


if __name__ == "__main__":
    sys.exit(main())
