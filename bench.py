"""Benchmark: BF16 GEMM TFLOP/s per GPU on B200 (headline config M=N=K=8192, TN).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One step = one launch of the persistent tcgen05 GEMM over the whole problem
(AUTO mode = 512x256 CTA-pair tiles here; bf16 in, fp32 accumulate, bf16 out). N=1 runs the 8192^3 square
GEMM of the square-sweep config (inputs N(0,1)*0.1 from seed 1). N>1 is
N-sharded weak scaling: every rank owns an 8192-column shard of an
M=8192, N=8192*world, K=8192 GEMM (A replicated, B rows = its output columns,
no collective inside the timed region), so the per-GPU problem equals the
N=1 problem. `value` = total FLOP of all ranks / max-over-ranks device time.

Inputs (A, B: 256 MiB) exceed the 126 MB L2, so no flush is needed between
steps. `e2e` times the same GEMM through the public plan API with the
operands copied from pinned host memory and D copied back every step.
`cpu_baseline` times the reference's CPU check path (fp32 einsum
"mkl,nkl->mnl", src/gemm/gemm_comparison.py:2705-2722) on a row slab of the
same operands using all host threads. `--impl reference` times that CPU path
alone as the reference arm.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
PKG_ROOT = REPO / "gb300-gemm-anatomy_b200"
for _p in (str(PKG_ROOT), str(REPO)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

M = N = K = 8192
METRIC = "BF16 GEMM TFLOP/s per GPU & % dense peak"
UNIT = "TFLOP/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic():
    """DRAM bytes per launch of the GEMM kernel from the committed ncu summary, if any."""
    p = REPO / "profiles" / "gemm_tn_sm100_8192_m512.md"
    if not p.is_file():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """SM clock and throttle-reason sampling during the timed region (NVML, else nvidia-smi)."""

    QUERY = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.t = None

    def _nvml_handle(self):
        """NVML handle of this process's CUDA device, matched by UUID (None if NVML is absent)."""
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(self.index).uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID("GPU-" + uuid)
        except Exception:  # noqa: BLE001 - any NVML problem falls back to nvidia-smi
            return None

    def _poll(self, nvml, handle):
        stop = self.stop_event
        while not stop.is_set():
            try:
                self.samples.append((time.time(),
                                     nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM),
                                     nvml.nvmlDeviceGetMaxClockInfo(handle, nvml.NVML_CLOCK_SM),
                                     nvml.nvmlDeviceGetCurrentClocksEventReasons(handle)))
            except Exception:  # noqa: BLE001
                break
            stop.wait(0.005)

    def start(self):
        # NVML read every 5 ms (read-only queries); nvidia-smi as the fallback
        # (or when B200_BENCH_CLOCKS=smi).
        got = None if os.environ.get("B200_BENCH_CLOCKS") == "smi" else self._nvml_handle()
        if got is not None:
            self.stop_event = threading.Event()
            self.samples = []
            self.t = threading.Thread(target=self._poll, args=got, daemon=True)
            self.nvml = got[0]
            self.t.start()
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def mark(self, which: str):
        """Wall-clock bounds of the timed region; only samples inside it are kept."""
        setattr(self, which, time.time())

    @staticmethod
    def _epoch(stamp: str):
        import datetime
        try:
            return datetime.datetime.strptime(stamp.strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            return None

    def _stop_nvml(self):
        self.stop_event.set()
        self.t.join(timeout=2)
        nvml = self.nvml
        bits = {"hw_slowdown": nvml.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": nvml.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": nvml.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": nvml.nvmlClocksEventReasonSwPowerCap}
        lo, hi = getattr(self, "t_start", None), getattr(self, "t_end", None)
        sm, mx, reasons = [], [], set()
        for ts, clk, clk_max, mask in self.samples:
            if lo is not None and hi is not None and not (lo <= ts <= hi):
                continue
            sm.append(float(clk))
            mx.append(float(clk_max))
            reasons.update(name for name, bit in bits.items() if mask & bit)
        try:
            nvml.nvmlShutdown()
        except Exception:  # noqa: BLE001
            pass
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvml, 5 ms"}

    def stop(self):
        if getattr(self, "nvml", None) is not None:
            return self._stop_nvml()
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.t is not None:
            self.t.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lo, hi = getattr(self, "t_start", None), getattr(self, "t_end", None)
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            ts = self._epoch(f[0])
            if lo is not None and hi is not None and ts is not None and not (lo <= ts <= hi):
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi"}


def cpu_reference_sample(a_cpu, b_cpu, budget_s: float):
    """Time the reference's CPU check math on a row slab sized to ~budget_s of work."""
    import torch
    from oracle import oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    # Grow the slab until one run costs a quarter of the budget, then scale to it.
    rows = 64
    while True:
        t0 = time.perf_counter()
        oracle.reference_einsum(a_cpu[:rows], b_cpu)
        probe = time.perf_counter() - t0
        if probe >= budget_s / 4 or rows >= a_cpu.shape[0]:
            break
        rows = min(a_cpu.shape[0], rows * 4)
    want = rows * budget_s / max(probe, 1e-4)
    reps = max(1, int(want // a_cpu.shape[0])) if want > a_cpu.shape[0] else 1
    rows = int(max(16, min(a_cpu.shape[0], want)))
    t0 = time.perf_counter()
    for _ in range(reps):
        oracle.reference_einsum(a_cpu[:rows], b_cpu)
    dt = time.perf_counter() - t0
    flop = 2.0 * rows * b_cpu.shape[0] * b_cpu.shape[1] * reps
    return flop / dt / 1e12, threads, rows * reps, dt


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference_arm(args):
    """CPU reference arm: the reference's fp32 CPU check path on this config."""
    import torch
    from b200gemm import operands

    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    a, b = operands.square_operands(M, seed=1)
    threads = os.cpu_count() or 1
    for _ in range(max(args.warmup, 0)):
        cpu_reference_sample(a, b, 0.25)
    vals, rows_used, secs = [], 0, 0.0
    for _ in range(args.steps):
        v, threads, rows_used, dt = cpu_reference_sample(a, b, 4.0)
        vals.append(v)
        secs += dt
    value = statistics.median(vals)
    sample = f"{rows_used} rows of A (M={M}) x full B (8192x8192), fp32 einsum, per step"
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": secs / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": f"gemm_tn {M}x{N}x{K} bf16 operands, fp32 CPU check path",
                   "m": M, "n": N, "k": K},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--mode", choices=["auto", "1cta", "2cta", "2cta_m512"], default="auto")
    ap.add_argument("--schedule", choices=["auto", "dynamic", "streamk"], default="auto",
                    help="tile schedule (auto: the library's choice)")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--cpu-budget-s", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        print("bench.py: --warmup must be >= 3", file=sys.stderr)
        return 2
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.schedule != "auto":
        os.environ["B200_GEMM_SCHEDULE"] = args.schedule  # read at plan creation

    import torch
    import torch.distributed as dist

    from b200gemm import gemm as G, operands

    world, rank, local = dist_env()
    if world != args.gpus:
        print(f"bench.py: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
        return 2
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    # Operands: A replicated; this rank's B shard (8192 rows of the global N = 8192*world).
    a_cpu, b0 = operands.square_operands(M, seed=1)
    if rank == 0:
        b_cpu = b0
    else:
        b_cpu = operands.normal_operands(N, 1, K, seed=1000 + rank, std_a=0.1, std_b=0.1)[0]
    a = a_cpu.to(dev)
    b = b_cpu.to(dev)
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)
    plan = G.GemmPlan(a, b, out, mode=args.mode, stream=stream)
    launches_per_step = plan.launches_per_execute
    schedule = plan.schedule

    for _ in range(args.warmup):
        plan.execute()
    plan.synchronize()

    peaks, peaks_kind = load_peaks()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    sampler.mark("t_start")
    ev0.record(stream)
    for _ in range(args.steps):
        plan.execute()
    ev1.record(stream)
    torch.cuda.synchronize()
    sampler.mark("t_end")
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    plan.synchronize()  # raises if any launch reported a device-side timeout
    ms_total = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms_total], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    ms_step = ms_total / args.steps
    flop_per_gpu = 2.0 * M * N * K
    value = flop_per_gpu * world / (ms_step / 1e3) / 1e12
    achieved = flop_per_gpu / (ms_step / 1e3) / 1e12  # one launch per step per GPU

    # End to end through the public API: every step uploads its operands from
    # pinned host memory, runs the GEMM and downloads D. The three parts use
    # different engines (H2D copy, SMs, D2H copy), so steps are pipelined over
    # three streams with double-buffered device operands: step i's upload
    # overlaps step i-1's GEMM and step i-2's download.
    a_pin = a_cpu.pin_memory()
    b_pin = b_cpu.pin_memory()
    d_pin = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
    s_in, s_comp, s_out = (torch.cuda.Stream(dev) for _ in range(3))
    bufs = [(a, b, out)] + [(torch.empty_like(a), torch.empty_like(b), torch.empty_like(out))]
    plans = [plan] + [G.GemmPlan(bufs[1][0], bufs[1][1], bufs[1][2], mode=args.mode, stream=s_comp)]
    ev = {name: [torch.cuda.Event() for _ in range(2)] for name in ("in", "comp", "out")}
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    s_comp.wait_event(e0)
    s_out.wait_event(e0)
    for i in range(args.e2e_steps):
        j = i % 2
        ai, bi, oi = bufs[j]
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(ev["comp"][j])   # step i-2's GEMM has read this set
            ai.copy_(a_pin, non_blocking=True)
            bi.copy_(b_pin, non_blocking=True)
            ev["in"][j].record(s_in)
        s_comp.wait_event(ev["in"][j])
        if i >= 2:
            s_comp.wait_event(ev["out"][j])      # step i-2's download has read this D
        plans[j].execute(s_comp)
        ev["comp"][j].record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev["comp"][j])
            d_pin.copy_(oi, non_blocking=True)
            ev["out"][j].record(s_out)
    e1.record(s_out)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    for pl in plans:
        pl.synchronize()
    e2e = {"value": flop_per_gpu * world / (e2e_ms / 1e3) / 1e12, "unit": UNIT,
           "h2d_bytes_per_step": (a.numel() + b.numel()) * 2, "d2h_bytes_per_step": out.numel() * 2,
           "ms_per_step": e2e_ms, "pipelined": "H2D / GEMM / D2H on three streams"}
    for pl in plans:
        pl.destroy()

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            v, threads, rows, dt = cpu_reference_sample(a_cpu, b_cpu, args.cpu_budget_s)
            cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                   "sample": f"{rows} rows of A (M={M}) x full B, fp32 einsum (reference CPU "
                             f"check path), {dt:.1f} s"}
        peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        traffic = profile_traffic()
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: A,B ~ N(0,1)*0.1 bf16 (seed 1; shard r>0 seed 1000+r)",
            "config": {"workload": f"gemm_tn {M}x{N * world}x{K} bf16->bf16, N-sharded "
                                   f"{N} cols/GPU" if world > 1 else f"gemm_tn {M}x{N}x{K} bf16->bf16",
                       "m": M, "n_per_gpu": N, "k": K, "mode": args.mode, "schedule": schedule,
                       "parallelism": f"n-shard x{world}", "l2": "inputs 256 MiB > L2, no flush"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": UNIT,
                         "frac": achieved / peak, "peak_kind": f"{peaks_kind} burst bf16",
                         "traffic": traffic},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": args.steps * launches_per_step,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
