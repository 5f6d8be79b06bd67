"""Stream-K schedule: tiles of the last wave split along K between clusters.

Parity of the split path through the C ABI, for both kernel shapes that run it
(1-CTA 128x256, pair 256x256) and both output types:
  integer operands (the reference's factory): fp32 D exact (max_abs_error 0);
  seeded uniform operands: the bf16 rule of the other GEMM tests against a
  float64 product, and fp32 D within 2^-20 * K of it (accumulation order only);
  repeated launches of one plan give identical bits (the partial flags are
  consumed and cleared inside every launch).
"""
import pytest
import torch

from b200gemm import check, gemm as G, operands

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def maxabs(t):
    return float(t.float().abs().max()) if t.numel() else 0.0


def plan_run(a_d, b_d, out_dtype, mode, repeats=1):
    out = torch.full((a_d.shape[0], b_d.shape[0]), float("nan"), dtype=out_dtype, device=DEV)
    plan = G.GemmPlan(a_d, b_d, out, mode=mode)
    try:
        sched = plan.schedule
        plan.execute()
        plan.synchronize()
        first = out.clone()
        for _ in range(repeats - 1):
            out.fill_(float("nan"))
            plan.execute()
        plan.synchronize()
        assert torch.equal(first, out), "repeated launches differ"
    finally:
        plan.destroy()
    return out, sched


# Shapes with an uneven last wave on a 148-SM B200 (1-CTA: 148 clusters of
# 128x256 tiles; pairs: 74 clusters), ragged edges, K that is not a whole
# number of 64-wide k-slices, and skinny grids (one side <= 4 blocks) where the
# clusters run in lanes and a tile is cut into up to four runs.
CASES = [
    ("1cta", (2560, 2048, 328)),       # 160 tiles over 148 CTAs
    ("1cta", (2500, 2000, 1024)),      # ragged M and N
    ("1cta", (8192, 512, 2048)),       # lanes along N (2), 64 m-blocks
    ("2cta", (2304, 2304, 520)),       # 81 tiles over 74 pairs
    ("2cta", (4096, 512, 1024)),       # lanes along N: 16 super-tiles over 37 groups
    ("2cta", (512, 8192, 4096)),       # lanes along M: 32 super-tiles over 37 groups
    ("2cta", (4000, 1304, 4096)),      # 96 tiles, ragged, long K
    ("2cta", (1000, 3000, 3000)),      # 4 m-blocks as lanes, ragged everything
    ("2cta", (5000, 2104, 200)),       # 180 tiles, ragged, 4 k-slices
    ("2cta", (16384, 512, 4096)),      # the reference's skinny frozen shape
    ("2cta", (512, 16384, 4096)),      # and its transpose
    ("2cta", (2304, 2304, 8)),         # one k-slice: some groups get no run at all
    ("2cta", (2304, 2304, 72)),        # two k-slices
    ("1cta", (4096, 512, 64)),         # lanes with a single k-slice
]


@pytest.mark.parametrize("mode,shape", CASES)
def test_stream_k_uniform(monkeypatch, mode, shape):
    monkeypatch.setenv("B200_GEMM_SCHEDULE", "streamk")
    m, n, k = shape
    a, b = operands.uniform_operands(m, n, k, seed=11)
    a_d, b_d = a.to(DEV), b.to(DEV)
    ref = (a_d.double() @ b_d.double().T).cpu()
    d, sched = plan_run(a_d, b_d, torch.bfloat16, mode, repeats=3)
    assert sched == "stream_k", f"{mode} {shape}: schedule {sched}"
    check.bf16_tolerance_check(f"{shape}/{mode}/sk", ref, d.cpu(), k, maxabs(a), maxabs(b))
    d32, _ = plan_run(a_d, b_d, torch.float32, mode, repeats=3)
    assert float((d32.cpu().double() - ref).abs().max()) <= 2.0 ** -20 * k


@pytest.mark.parametrize("mode", ["1cta", "2cta"])
def test_stream_k_integer_exact(monkeypatch, mode):
    monkeypatch.setenv("B200_GEMM_SCHEDULE", "streamk")
    m, n, k = {"1cta": (2560, 2048, 1024), "2cta": (2304, 2304, 1024)}[mode]
    a, b = operands.integer_operands(m, n, k)
    a_d, b_d = a.to(DEV), b.to(DEV)
    d, sched = plan_run(a_d, b_d, torch.float32, mode, repeats=2)
    assert sched == "stream_k"
    ref = a_d.float() @ b_d.float().T  # integer products and sums: exact in fp32
    assert torch.equal(d, ref)


def test_two_accumulator_tiles_stay_dynamic(monkeypatch):
    """512 x 256 pair tiles fill both TMEM slots: even when forced they keep the dynamic schedule."""
    monkeypatch.setenv("B200_GEMM_SCHEDULE", "streamk")
    m, n, k = 4608, 2304, 1024
    a, b = operands.integer_operands(m, n, k)
    a_d, b_d = a.to(DEV), b.to(DEV)
    d, sched = plan_run(a_d, b_d, torch.float32, "2cta_m512")
    assert sched == "dynamic"
    assert torch.equal(d, a_d.float() @ b_d.float().T)


def test_auto_picks_stream_k_on_an_uneven_last_wave(monkeypatch):
    """4096^3 on 74 pairs: 256 tiles = 3.46 waves -> stream-K; 8192^2 x 512 -> dynamic."""
    monkeypatch.delenv("B200_GEMM_SCHEDULE", raising=False)
    if torch.cuda.get_device_properties(0).multi_processor_count != 148:
        pytest.skip("schedule thresholds are stated for a 148-SM B200")
    a, b = operands.uniform_operands(4096, 4096, 4096, seed=12)
    a_d, b_d = a.to(DEV), b.to(DEV)
    d_sk, sched = plan_run(a_d, b_d, torch.bfloat16, "auto")
    assert sched == "stream_k"
    monkeypatch.setenv("B200_GEMM_SCHEDULE", "dynamic")
    d_dyn, sched = plan_run(a_d, b_d, torch.bfloat16, "auto")
    assert sched == "dynamic"
    ref = (a_d.double() @ b_d.double().T).cpu()
    check.bf16_tolerance_check("4096^3/sk", ref, d_sk.cpu(), 4096, maxabs(a), maxabs(b))
    check.bf16_tolerance_check("4096^3/dyn", ref, d_dyn.cpu(), 4096, maxabs(a), maxabs(b))
    monkeypatch.delenv("B200_GEMM_SCHEDULE")
    a2, b2 = operands.uniform_operands(8192, 8192, 512, seed=13)
    out = torch.empty((8192, 8192), dtype=torch.bfloat16, device=DEV)
    plan = G.GemmPlan(a2.to(DEV), b2.to(DEV), out)
    try:
        assert plan.schedule == "dynamic"  # 32 x 32 tiles of 256 x 256 / 74 = 13.8 waves
    finally:
        plan.destroy()


def test_stream_k_back_to_back_launches(monkeypatch):
    """Launches queued without a host sync (PDL overlaps their setup): same bits every time."""
    monkeypatch.setenv("B200_GEMM_SCHEDULE", "streamk")
    m, n, k = 2304, 2304, 2048
    a, b = operands.uniform_operands(m, n, k, seed=14)
    a_d, b_d = a.to(DEV), b.to(DEV)
    outs = [torch.empty((m, n), dtype=torch.float32, device=DEV) for _ in range(2)]
    plans = [G.GemmPlan(a_d, b_d, o, mode="2cta") for o in outs]
    try:
        assert all(p.schedule == "stream_k" for p in plans)
        for i in range(20):
            plans[i % 2].execute()
        plans[0].synchronize()
        plans[1].synchronize()
    finally:
        for p in plans:
            p.destroy()
    assert torch.equal(outs[0], outs[1])
    ref = a_d.double() @ b_d.double().T
    assert float((outs[0].double() - ref).abs().max()) <= 2.0 ** -20 * k


def _random_cases(count=24, seed=2024):
    import random
    rng = random.Random(seed)
    cases = []
    while len(cases) < count:
        mode = rng.choice(["1cta", "2cta"])
        m = rng.randrange(64, 6144, 8)
        n = rng.randrange(64, 4096, 8)
        k = rng.randrange(64, 3072, 8)
        cases.append((mode, (m, n, k)))
    return cases


@pytest.mark.parametrize("mode,shape", _random_cases())
def test_stream_k_random_shapes(monkeypatch, mode, shape):
    """Seeded random shapes, stream-K forced: every split layout the walk produces is exact
    up to accumulation order (fp32 D within 2^-20 * K of the float64 product)."""
    monkeypatch.setenv("B200_GEMM_SCHEDULE", "streamk")
    m, n, k = shape
    a, b = operands.uniform_operands(m, n, k, seed=m + n + k)
    a_d, b_d = a.to(DEV), b.to(DEV)
    d, _ = plan_run(a_d, b_d, torch.float32, mode, repeats=2)
    ref = a_d.double() @ b_d.double().T
    assert float((d.double() - ref).abs().max()) <= 2.0 ** -20 * k


@pytest.mark.parametrize("shape", [(8192, 8192, 8192), (4096, 4096, 4096), (16384, 512, 4096),
                                   (32768, 512, 4096), (512, 512, 512), (8192, 1792, 4096),
                                   (8192, 4096, 4096)])
def test_policy_preview_matches_plans(shape):
    """b200_gemm_policy (no device) predicts what plan creation on this GPU decides."""
    m, n, k = shape
    sm = torch.cuda.get_device_properties(0).multi_processor_count
    pred = G.policy(m, n, k, sm_count=sm)
    a = torch.empty((m, k), dtype=torch.bfloat16, device=DEV)
    b = torch.empty((n, k), dtype=torch.bfloat16, device=DEV)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=DEV)
    plan = G.GemmPlan(a, b, out)
    try:
        info = plan.info
        assert pred["schedule"] == plan.schedule
        assert pred["num_tiles"] == info["num_tiles"]
        assert pred["grid_ctas"] == info["grid_ctas"]
        assert pred["tile_m"] == info["tile_m"]
    finally:
        plan.destroy()


_PARTIAL_RESIDENCY_CHILD = r"""
import sys, time
sys.path.insert(0, "gb300-gemm-anatomy_b200")
import torch
from b200gemm import _lib, gemm as G, operands
torch.backends.cuda.matmul.allow_tf32 = False
dev = torch.device("cuda", 0)
lib = _lib.load()
a, b = operands.integer_operands(4096, 4096, 4096, seed=31)
a, b = a.to(dev), b.to(dev)
ref = a.float() @ b.float().T
sms = torch.cuda.get_device_properties(dev).multi_processor_count
s_other, s_gemm = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
out = torch.full((4096, 4096), float("nan"), dtype=torch.float32, device=dev)
plan = G.GemmPlan(a, b, out, mode="auto", stream=s_gemm)
assert plan.schedule == "stream_k", plan.schedule
for hold_ms in (1500, 0):
    out.fill_(float("nan"))
    torch.cuda.synchronize()
    if hold_ms:
        # Another tenant holds half of the SMs for longer than the wait limit.
        rc = lib.b200_selftest_occupy(sms // 2, 200 * 1024, hold_ms * 1000000, s_other.cuda_stream)
        assert rc == 0, _lib.last_error()
        time.sleep(0.05)
    t0 = time.perf_counter()
    plan.execute()
    plan.synchronize()
    torch.cuda.synchronize()
    print("ELAPSED", hold_ms, time.perf_counter() - t0)
    print("MAXERR", hold_ms, float((out - ref).abs().max()))
plan.destroy()
"""


def test_stream_k_completes_with_half_the_sms_taken():
    """A stream-K launch that finds only part of its clusters resident still
    finishes and is exact: finishers only wait for lower-numbered clusters.

    Another kernel holds half the SMs for 1.5 s while the wait limit is 0.4 s,
    so a finisher that waited for a cluster which cannot start yet would report
    0x108 instead. Runs in a child process (the wait limit is read once per
    process)."""
    import os
    import subprocess
    import sys
    from pathlib import Path
    env = dict(os.environ, B200_WAIT_TIMEOUT_MS="400")
    env.pop("B200_GEMM_SCHEDULE", None)
    root = Path(__file__).resolve().parents[1]
    res = subprocess.run([sys.executable, "-c", _PARTIAL_RESIDENCY_CHILD], cwd=root, env=env,
                         capture_output=True, text=True, timeout=180)
    assert res.returncode == 0, res.stderr[-3000:]
    errs = [float(line.split()[2]) for line in res.stdout.splitlines() if line.startswith("MAXERR")]
    assert errs == [0.0, 0.0], res.stdout
