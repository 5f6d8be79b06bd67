"""The drivers end to end on the GPU (reference-compatible command lines)."""
import csv
import io
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parents[1]


def run(mod, *args, timeout=600):
    env = dict(os.environ, PYTHONPATH=str(REPO / "gb300-gemm-anatomy_b200") + os.pathsep + str(REPO))
    return subprocess.run([sys.executable, "-m", mod, *args], capture_output=True, text=True,
                          env=env, timeout=timeout)


def test_gemm_comparison_ref_compat_exact():
    r = run("b200gemm.cli.gemm_comparison", "--shape", "512x512x512", "--shape", "256x1024x768",
            "--iterations", "3", "--warmup-iterations", "1",
            "--candidates", "persistent_1cta,persistent_2cta,torch_matmul")
    assert r.returncode == 0, r.stderr
    rows = list(csv.DictReader(io.StringIO(r.stdout)))
    assert len(rows) == 6
    for row in rows:
        assert row["correctness"] == "PASS"
        if row["method"] == "b200":
            assert float(row["max_abs_error"]) == 0.0  # integer operands: exact, like the reference
        assert float(row["tflops"]) > 0


def test_gemm_comparison_bf16_config_operands():
    r = run("b200gemm.cli.gemm_comparison", "--shapes", "c1", "--operands", "config",
            "--out-dtype", "bf16", "--iterations", "3", "--warmup-iterations", "1",
            "--candidates", "persistent_1cta,persistent_2cta")
    assert r.returncode == 0, r.stderr
    rows = list(csv.DictReader(io.StringIO(r.stdout)))
    assert [row["variant"] for row in rows] == ["persistent_1cta", "persistent_2cta"]
    assert all(float(row["max_rel_error"]) <= 1e-2 for row in rows)


def test_memory_paths_self_test():
    r = run("b200gemm.cli.memory_paths", "--self-test")
    assert r.returncode == 0, r.stderr
    assert "SELF_TEST_RESULT=PASS" in r.stderr


def test_memory_paths_uniform_checksum_run():
    r = run("b200gemm.cli.memory_paths", "--method", "tma_sw128", "--stages", "4",
            "--stage-kib", "16", "--ctas-per-sm", "2", "--working-set-mib", "300",
            "--run-kind", "benchmark", "--fill", "uniform", "--repetitions", "2",
            "--warmup-ms", "10")
    assert r.returncode == 0, r.stderr
    rows = list(csv.DictReader(io.StringIO(r.stdout)))
    assert len(rows) == 2
    assert rows[0]["checksum_xor"] == rows[0]["host_checksum_xor"]
    assert rows[0]["checksum_sum"] == rows[0]["host_checksum_sum"]
    assert float(rows[0]["effective_gbps"]) > 100


def test_umma_self_test():
    r = run("b200gemm.cli.umma", "--self-test")
    assert r.returncode == 0, r.stderr


def test_umma_timed_row():
    r = run("b200gemm.cli.umma", "--mode", "2sm", "--n", "256", "--depth", "64",
            "--iterations", "100", "--repetitions", "2", "--warmup", "1")
    assert r.returncode == 0, r.stderr
    rows = list(csv.DictReader(io.StringIO(r.stdout)))
    assert len(rows) == 2 and float(rows[0]["flops_per_cycle_per_sm"]) > 1000


def test_sharded_gemm_single_rank_gather():
    sys.path.insert(0, str(REPO / "gb300-gemm-anatomy_b200"))
    from b200gemm import dist as bdist, operands
    dev = torch.device("cuda", 0)
    a, b = operands.uniform_operands(256, 200, 128, seed=3)
    sg = bdist.ShardedGemm(a.to(dev), b.to(dev), 200, out_dtype=torch.float32)
    full = sg.run("full")
    sg.synchronize()
    sg.destroy()
    ref = a.float() @ b.float().T
    assert float((full.cpu() - ref).abs().max()) <= 1e-3
