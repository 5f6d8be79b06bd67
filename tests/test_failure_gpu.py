"""Failure detection on the GPU without faulting it.

A kernel waits on an mbarrier that nothing arrives on; its bounded wait must
give up within the budget, report B200_DEV_TIMEOUT_SELFTEST through the status
word, and leave the context usable (a GEMM right after still succeeds).
"""
import time

import pytest
import torch

from b200gemm import _lib, gemm as G, operands

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    t0 = time.perf_counter()
    rc = lib.b200_selftest_bounded_wait(20_000_000, status.data_ptr(),
                                        torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.OK, _lib.last_error()
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(status.item()) == 0x107
    assert elapsed < 5.0
    a, b = operands.uniform_operands(256, 256, 128, seed=1)
    out = G.gemm(a.to(dev), b.to(dev))
    ref = a.float() @ b.float().T
    assert float((out.cpu().float() - ref).abs().max()) < 0.1


def test_bounded_wait_argument_checks():
    lib = _lib.load()
    assert lib.b200_selftest_bounded_wait(0, 16, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.b200_selftest_bounded_wait(1000, None, None) == _lib.ERR_INVALID_ARGUMENT


_DROP_FLAGS_CHILD = r"""
import sys, time
sys.path.insert(0, "gb300-gemm-anatomy_b200")
import os, torch
from b200gemm import _lib, gemm as G, operands
dev = torch.device("cuda", 0)
a, b = operands.uniform_operands(2304, 2304, 1024, seed=21)
a, b = a.to(dev), b.to(dev)
out = torch.empty((2304, 2304), dtype=torch.float32, device=dev)
plan = G.GemmPlan(a, b, out, mode="2cta")
assert plan.schedule == "stream_k", plan.schedule
t0 = time.perf_counter()
plan.execute()
try:
    plan.synchronize()
    print("NO_TIMEOUT")
except _lib.BridgeError as exc:
    print("ELAPSED", time.perf_counter() - t0)
    print("CODE", exc.code)
    print("MSG", str(exc))
plan.destroy()
del os.environ["B200_TEST_DROP_PARTIAL_FLAGS"]
plan = G.GemmPlan(a, b, out, mode="2cta")
plan.execute()
plan.synchronize()
plan.destroy()
ref = a.double() @ b.double().T
print("AFTER_MAXERR", float((out.double() - ref).abs().max()))
"""


def test_stream_k_partial_wait_times_out_and_context_survives():
    """Partial writers that never set their flag: finishers give up with 0x108, no hang.

    Runs in a child process: the wait limit (B200_WAIT_TIMEOUT_MS, 200 ms here)
    is read once per process.
    """
    import os
    import subprocess
    import sys
    from pathlib import Path
    env = dict(os.environ, B200_WAIT_TIMEOUT_MS="200", B200_GEMM_SCHEDULE="streamk",
               B200_TEST_DROP_PARTIAL_FLAGS="1")
    root = Path(__file__).resolve().parents[1]
    res = subprocess.run([sys.executable, "-c", _DROP_FLAGS_CHILD], cwd=root, env=env,
                         capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = dict(line.split(" ", 1) for line in res.stdout.strip().splitlines() if " " in line)
    assert "NO_TIMEOUT" not in res.stdout
    assert int(lines["CODE"]) == _lib.ERR_DEVICE_TIMEOUT
    assert "0x108" in lines["MSG"]
    assert float(lines["ELAPSED"]) < 10.0
    assert float(lines["AFTER_MAXERR"]) <= 2.0 ** -20 * 1024
