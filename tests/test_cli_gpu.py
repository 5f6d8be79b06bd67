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


def _golden_headers():
    import json
    return json.loads((REPO / "tests" / "golden" / "row_contracts.json").read_text())


def test_gemm_comparison_p35_schema_rows():
    """--schema p35: exactly the reference's 100 columns, its value conventions
    (not_applicable markers, fixed-point reals), the reference's own cuBLASLt bridge
    row with its plan metadata when the bridge is built."""
    cands = "persistent_auto,persistent_2cta,torch_matmul"
    bridge = (REPO / "baseline" / "_ref" / "libcublaslt_bridge_p35.so").is_file()
    if bridge:
        cands += ",heuristic_first_supported"
    r = run("b200gemm.cli.gemm_comparison", "--shape", "4096x4096x4096", "--schema", "p35",
            "--iterations", "3", "--warmup-iterations", "1", "--candidates", cands)
    assert r.returncode == 0, r.stderr
    header = r.stdout.splitlines()[0].split(",")
    assert header == _golden_headers()["p35"]
    rows = list(csv.DictReader(io.StringIO(r.stdout)))
    assert all(len(row) == 100 and "" not in row.values() for row in rows)
    by = {row["variant"]: row for row in rows}
    auto = by["persistent_auto"]
    assert auto["scheduler"] == "stream_k_persistent" and auto["algo_id"] == "not_applicable"
    assert auto["max_abs_error"] == "0.000000000" and auto["use_tma_store"] == "true"
    assert int(auto["max_active_clusters"]) >= 1 and len(auto["upstream_kernel_sha256"]) == 64
    assert by["persistent_2cta"]["best_cutedsl_variant"] in ("persistent_auto", "persistent_2cta")
    assert by["torch_matmul"]["scheduler"] == "not_applicable"
    assert auto["gpu_uuid"].startswith("GPU-")
    if bridge:
        lt = by["heuristic_first_supported"]
        assert lt["order_a"] == "CUBLASLT_ORDER_ROW" and int(lt["algo_id"]) >= 0
        assert lt["lda"] == "4096" and lt["scheduler"] == "not_applicable"


def test_memory_and_umma_reference_schema_rows():
    r = run("b200gemm.cli.memory_paths", "--method", "ldgsts", "--stages", "2",
            "--stage-kib", "16", "--working-set-mib", "300", "--run-kind", "benchmark",
            "--repetitions", "1", "--warmup-ms", "5", "--schema", "ref")
    assert r.returncode == 0, r.stderr
    g = _golden_headers()
    assert r.stdout.splitlines()[0].split(",") == g["memory"]["ldgsts"]
    row = next(csv.DictReader(io.StringIO(r.stdout)))
    assert row["copies_per_thread_per_stage"] == "8" and row["gpu_uuid"].startswith("GPU-")
    assert int(row["cuda_driver_version"]) > 0 and row["correctness"] == "OK"
    r = run("b200gemm.cli.umma", "--mode", "2sm", "--n", "128", "--depth", "16",
            "--iterations", "10", "--repetitions", "1", "--warmup", "1", "--schema", "ref")
    assert r.returncode == 0, r.stderr
    assert r.stdout.splitlines()[0].split(",") == g["umma"]["umma_2sm"]
    row = next(csv.DictReader(io.StringIO(r.stdout)))
    assert row["method"] == "umma_2sm" and row["total_umma"] == "160"
    assert row["flops_per_umma"] == str(2 * 256 * 128 * 16) and row["max_abs_error"] == "0.000000"


def test_gemm_comparison_cutedsl_context_rows():
    """NVIDIA's CuTe DSL examples as context candidates beside ours (fp32 D,
    integer operands: every candidate exact)."""
    sys.path.insert(0, str(REPO / "gb300-gemm-anatomy_b200"))
    from b200gemm.cli import cutedsl_baseline
    ok, why = cutedsl_baseline.available()
    if not ok:
        pytest.skip(why)
    r = run("b200gemm.cli.gemm_comparison", "--shape", "1024x512x256", "--iterations", "2",
            "--warmup-iterations", "1", "--candidates",
            "persistent_auto,cutedsl_nonpersistent_1cta,cutedsl_persistent_1cta,"
            "cutedsl_persistent_2cta", timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]
    rows = list(csv.DictReader(io.StringIO(r.stdout)))
    assert [row["method"] for row in rows] == ["b200", "cutedsl", "cutedsl", "cutedsl"]
    for row in rows:
        assert float(row["max_abs_error"]) == 0.0
    assert rows[3]["use_2cta_instrs"] == "true" and rows[3]["mma_tiler_m"] == "256"
    assert float(rows[2]["compile_time_ms"]) > 0 and rows[1]["max_active_clusters"] == "not_applicable"
    assert rows[0]["best_cutedsl_variant"].startswith("cutedsl_")
