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

Further sections of the same JSON line (after the headline's timed region;
`--no-extras` skips them):
  llm_shard    (every N) config c5, 8192 x {128256, 14336} x 4096, N split over
               the ranks (strong scaling), gathers none / fused / fused_mc / nccl, each
               checked on every rank against torch IEEE fp32 on 64 sampled rows
               before it is timed (max over ranks)
  sustained    (N=1) >= 2 s windows of back-to-back 8192^3 launches, ours and
               cuBLAS alternated, median SM clock and power per window (NVML),
               frac against the measured sustained bf16 peak
  memory_path  (N=1) config c2: 4 GiB streamed by TMA and LDGSTS, device
               checksum == host checksum, GB/s against the measured HBM copy
               peak, and the CPU streaming-checksum baseline on all host cores
  umma         (N=1) config c3: 2-SM tcgen05.mma N=256 depth 256 on all SMs,
               exact known answer, FLOP/cycle/SM
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
                                     nvml.nvmlDeviceGetCurrentClocksEventReasons(handle),
                                     nvml.nvmlDeviceGetPowerUsage(handle) / 1000.0))
            except Exception:  # noqa: BLE001
                break
            stop.wait(0.001)

    def start(self):
        # NVML read every 1 ms (read-only queries); nvidia-smi as the fallback
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

    def window(self, lo: float, hi: float):
        """Median SM clock, median power and throttle reasons of the NVML samples in [lo, hi]."""
        nvml = self.nvml
        bits = {"hw_slowdown": nvml.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": nvml.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": nvml.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": nvml.nvmlClocksEventReasonSwPowerCap}
        sm, pw, reasons = [], [], set()
        for ts, clk, _, mask, watts in list(self.samples):
            if lo <= ts <= hi:
                sm.append(float(clk))
                pw.append(float(watts))
                reasons.update(name for name, bit in bits.items() if mask & bit)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "power_w": statistics.median(pw) if pw else None,
                "reasons": sorted(reasons), "samples": len(sm)}

    def _stop_nvml(self):
        self.stop_event.set()
        self.t.join(timeout=2)
        nvml = self.nvml
        bits = {"hw_slowdown": nvml.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": nvml.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": nvml.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": nvml.nvmlClocksEventReasonSwPowerCap}
        lo, hi = getattr(self, "t_start", None), getattr(self, "t_end", None)
        samples = self.samples
        if lo is not None and hi is not None:
            inside = [x for x in samples if lo <= x[0] <= hi]
            if not inside and samples:
                # A timed region shorter than the polling gap: the sample closest to it.
                inside = [min(samples, key=lambda x: min(abs(x[0] - lo), abs(x[0] - hi)))]
            samples = inside
        sm, mx, reasons = [], [], set()
        for ts, clk, clk_max, mask, _ in samples:
            sm.append(float(clk))
            mx.append(float(clk_max))
            reasons.update(name for name, bit in bits.items() if mask & bit)
        try:
            nvml.nvmlShutdown()
        except Exception:  # noqa: BLE001
            pass
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvml, 1 ms"}

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


def _event_ms(fn, iters, stream):
    """CUDA-event time of `iters` back-to-back calls of fn() on `stream`, in ms per call."""
    import torch
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(iters):
        fn()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / iters


def sustained_section(plan, a, b, local, peaks, seconds: float = 2.0):
    """Back-to-back 8192^3 launches for `seconds` each, ours and cuBLAS alternated
    twice, with NVML clock and power over each window: steady operation under
    the 1000 W cap rather than the short headline burst."""
    import torch

    stream = torch.cuda.current_stream()
    flop = 2.0 * a.shape[0] * b.shape[0] * a.shape[1]
    c = torch.empty((a.shape[0], b.shape[0]), dtype=torch.bfloat16, device=a.device)
    bt = b.t()
    impls = {"b200": plan.execute, "cublas": lambda: torch.mm(a, bt, out=c)}
    per_launch = {}
    for name, fn in impls.items():  # launches per window from a short probe
        fn()
        per_launch[name] = _event_ms(fn, 20, stream)
    sampler = ClockSampler(local)
    sampler.start()
    has_nvml = getattr(sampler, "nvml", None) is not None
    time.sleep(0.2)
    runs = {"b200": [], "cublas": []}
    for _ in range(2):
        for name, fn in impls.items():
            n = max(1, int(seconds * 1e3 / per_launch[name]))
            torch.cuda.synchronize()
            t0 = time.time()
            ms = _event_ms(fn, n, stream)
            t1 = time.time()
            win = sampler.window(t0, t1) if has_nvml else {}
            runs[name].append({"tflops": flop / (ms / 1e3) / 1e12, "launches": n,
                               "seconds": n * ms / 1e3, **win})
    sampler.stop()
    plan.synchronize()
    peak = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    out = {"workload": "gemm_tn 8192x8192x8192 bf16->bf16, back to back", "unit": UNIT,
           "peak": peak, "peak_kind": "bf16_tflops_sustained"}
    for name, rs in runs.items():
        v = statistics.median(r["tflops"] for r in rs)
        out[name] = {"tflops": v, "frac": v / peak, "windows": rs}
    if has_nvml:
        for name in runs:
            pw = [r["power_w"] for r in runs[name] if r.get("power_w")]
            if pw:
                out[name]["tflops_per_joule"] = out[name]["tflops"] / statistics.median(pw)
    return out


def llm_shard_section(world, rank, dev, shapes=((128256, 4096), (14336, 4096)), m=8192,
                      iters=10, warmup=3):
    """Config c5 N-sharded over the ranks (strong scaling: N fixed, split by
    b200_shard_range), each gather timed: none (the shard GEMM alone), fused
    (the GEMM epilogue stores every output chunk into every rank's full D over
    NVLink), fused_mc (the same through an NVLink multicast address: one store,
    replicated by the switch) and nccl (GEMM, then NCCL all-gather + re-layout). Before timing,
    every rank checks the full gathered D (its own shard with gather none) on
    64 sampled rows against torch's IEEE fp32 matmul with the bf16 rule;
    the results are combined over ranks."""
    import torch
    import torch.distributed as dist

    from b200gemm import check, dist as bdist, operands

    torch.backends.cuda.matmul.allow_tf32 = False
    gathers = ("none", "fused", "fused_mc", "nccl") if world > 1 else ("none",)
    out = {"operands": "c5: A ~ N(0,1), B ~ N(0,0.02), seed 2, drawn on the device",
           "scaling": "strong: N fixed, split over the ranks", "check_rows": 64, "shapes": {}}
    for (n, k) in shapes:
        a, b_full = operands.llm_operands_device(n, k, dev, m=m)
        n0, n1 = bdist.shard_bounds(n, world, rank)
        b = b_full[n0:n1].contiguous()
        rows = torch.arange(0, m, m // 64, device=dev)
        ref = a[rows].float() @ b_full.float().t()
        amax, bmax = float(a.float().abs().max()), float(b_full.float().abs().max())
        del b_full
        res = {"shard_cols": n1 - n0}
        for gather in gathers:
            try:
                sg = bdist.ShardedGemm(a, b, n, p2p=gather.startswith("fused"),
                                       engine="mc" if gather == "fused_mc" else "sm")
            except Exception as exc:  # noqa: BLE001 - e.g. no NVLink multicast on this node
                res[gather] = {"unavailable": str(exc)}
                continue
            mode = "none" if gather == "none" else "full"
            got = sg.run(mode)
            torch.cuda.synchronize()
            want = ref if gather != "none" else ref[:, n0:n1]
            ok = 1
            try:
                check.bf16_tolerance_check(f"{m}x{n}x{k} {gather}", want, got[rows].float(), k, amax, bmax)
            except check.CorrectnessError as exc:
                print(f"bench.py: llm_shard check failed on rank {rank}: {exc}", file=sys.stderr)
                ok = 0
            del got
            for _ in range(warmup):
                sg.run(mode)
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            ms = _event_ms(lambda: sg.run(mode), iters, torch.cuda.current_stream())
            sg.synchronize()
            t = torch.tensor([ms, -ok], dtype=torch.float64, device=dev)
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)  # slowest rank; any failed check
            sg.destroy()
            ms = float(t[0])
            entry = {"ms": ms, "tflops": 2.0 * m * n * k / (ms / 1e3) / 1e12,
                     "check": "pass" if float(t[1]) < 0 else "FAIL"}
            if gather != "none":
                sent = m * (n1 - n0) * 2 * (world - 1)
                entry["sent_gbps_per_gpu"] = sent / (ms / 1e3) / 1e9
            res[gather] = entry
            torch.cuda.empty_cache()
        out["shapes"][f"{m}x{n}x{k}"] = res
        del a, b, ref
        torch.cuda.empty_cache()
    return out


def _parallel_checksum(words, threads):
    """XOR and 64-bit sum of a uint32 array on `threads` host threads (numpy
    reductions release the GIL)."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor

    parts = np.array_split(words, threads * 4)

    def one(w):
        return int(np.bitwise_xor.reduce(w)) if w.size else 0, int(w.sum(dtype=np.uint64))

    with ThreadPoolExecutor(max_workers=threads) as pool:
        res = list(pool.map(one, parts))
    x = 0
    tot = 0
    for px, ps in res:
        x ^= px
        tot = (tot + ps) & ((1 << 64) - 1)
    return x, tot


def memory_path_section(dev, peaks, nbytes=4 << 30, reps=5):
    """Config c2: a 4 GiB seeded bf16 buffer streamed HBM -> SMEM by TMA and by
    LDGSTS (best configurations of the sweep, and the best of the reference's
    1-CTA/SM grid). Each first checksums the buffer on the device (must equal
    the host checksum bit for bit), then is timed in the reference's sink mode:
    GB/s = working set / kernel time (src/memory/ldgsts.cu:898,913-916). The CPU
    baseline streams the same bytes through an XOR + 64-bit sum on all host cores."""
    import argparse as _ap

    import numpy as np
    import torch

    from b200gemm.cli import memory_paths as cmp

    g = torch.Generator(device=dev).manual_seed(2)
    buf = torch.empty(nbytes // 2, dtype=torch.bfloat16, device=dev)
    chunk = 1 << 28
    for i in range(0, buf.numel(), chunk):
        buf[i:i + chunk] = torch.rand(min(chunk, buf.numel() - i), generator=g, device=dev) * 2 - 1
    words = buf.view(torch.int32).cpu().numpy().view(np.uint32)
    threads = os.cpu_count() or 1
    _parallel_checksum(words[: 1 << 24], threads)  # warm the pool
    cpu_times, host = [], None
    for _ in range(3):
        t0 = time.perf_counter()
        host = _parallel_checksum(words, threads)
        cpu_times.append(time.perf_counter() - t0)
    cmp._HOST_CHECKSUMS[(buf.data_ptr(), nbytes)] = host
    del words
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    args = _ap.Namespace(fill="uniform", warmup_ms=100, repetitions=reps, passes=1,
                         run_kind="benchmark")
    configs = [("best_tma", "tma_sw128", 2, 16384, 4), ("best_ldgsts", "ldgsts", 2, 16384, 4),
               ("ref_grid_tma", "tma", 2, 32768, 1), ("ref_grid_ldgsts", "ldgsts", 2, 32768, 1)]
    out = {"workload": f"{nbytes >> 30} GiB seeded uniform bf16, HBM -> SMEM, 1 pass", "unit": "GB/s",
           "peak": hbm, "peak_kind": "hbm_gbs (measured copy)"}
    for label, method, stages, sb, ctas in configs:
        rows = cmp.run_one(buf, method, stages, sb, ctas, args, nbytes, hbm)
        gbps = [r["effective_gbps"] for r in rows]
        out[label] = {"method": method, "stages": stages, "stage_bytes": sb, "ctas_per_sm": ctas,
                      "gbps_best": max(gbps), "gbps_median": statistics.median(gbps),
                      "frac": max(gbps) / hbm, "checksum": "device == host",
                      "checksum_xor": rows[0]["checksum_xor"], "checksum_sum": rows[0]["checksum_sum"]}
    out["cpu_baseline"] = {"gbps": nbytes / min(cpu_times) / 1e9, "unit": "GB/s", "cores": threads,
                           "kind": "XOR + 64-bit sum of every 32-bit word, numpy on host threads",
                           "sample": f"the same {nbytes >> 30} GiB, best of 3"}
    del buf
    torch.cuda.empty_cache()
    return out


def umma_section(reps=5):
    """Config c3: tcgen05.mma 2-SM (cta_group::2), M=256 N=256 K=16, depth 256,
    one CTA pair on every SM pair, 1000 commit rounds; the integer known answer
    is checked exactly first (src/compute/umma_1sm.cu:577-586, 1164-1167)."""
    import argparse as _ap

    import torch

    from b200gemm.cli import umma as cu

    sms = torch.cuda.get_device_properties(0).multi_processor_count
    args = _ap.Namespace(operands="pattern", iterations=1000, warmup=3, repetitions=reps,
                         self_test=False)
    rows = cu.run_case(2, 256, 256, args, sms // 2, sms, "umma_2sm")
    fpc = [r["flops_per_cycle_per_sm"] for r in rows]
    tf = [r["tflops"] for r in rows]
    return {"workload": "umma_2sm N=256 depth=256 x 1000 iterations, all SMs", "check": "exact",
            "flops_per_cycle_per_sm": statistics.median(fpc), "ceiling_flops_per_cycle_per_sm": 8192,
            "frac": statistics.median(fpc) / 8192, "tflops_all_sms": statistics.median(tf)}


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
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the llm_shard, sustained, memory_path and umma sections")
    ap.add_argument("--sustained-s", type=float, default=2.0,
                    help="seconds per window of the sustained section (two windows per impl)")
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
    for pl in plans[1:]:
        pl.destroy()
    del bufs, plans, a_pin, b_pin, d_pin

    extras = {}
    if not args.no_extras:
        if world == 1:
            extras["sustained"] = sustained_section(plan, a, b, local, peaks, args.sustained_s)
        plan.destroy()
        del a, b, out
        torch.cuda.empty_cache()
        extras["llm_shard"] = llm_shard_section(world, rank, dev)
        if world == 1:
            extras["memory_path"] = memory_path_section(dev, peaks)
            extras["umma"] = umma_section()
    else:
        plan.destroy()

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
            **extras,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
