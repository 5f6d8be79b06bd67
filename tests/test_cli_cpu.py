"""Command-line contracts of the drivers without a GPU (exit codes, self-test)."""
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
ENV_PATH = str(REPO / "gb300-gemm-anatomy_b200")


def run(mod, *args):
    import os
    env = dict(os.environ, PYTHONPATH=ENV_PATH + os.pathsep + str(REPO), CUDA_VISIBLE_DEVICES="")
    return subprocess.run([sys.executable, "-m", mod, *args], capture_output=True, text=True,
                          env=env, timeout=120)


def test_gemm_comparison_self_test():
    r = run("b200gemm.cli.gemm_comparison", "--self-test")
    assert r.returncode == 0 and "SELF_TEST_RESULT=PASS" in r.stderr and r.stdout == ""


@pytest.mark.parametrize("args", [["--iterations", "0"], ["--iterations", "101"],
                                  ["--warmup-iterations", "abc"], ["--shape", "8x8"],
                                  ["--candidates", "nope"], ["--schedule", "fast"]])
def test_gemm_comparison_usage_errors(args):
    r = run("b200gemm.cli.gemm_comparison", *args)
    assert r.returncode == 2 and r.stdout == ""


@pytest.mark.parametrize("args", [["--stages", "3"], ["--stages", "4"],
                                  ["--stages", "4", "--bytes-in-flight-kib", "64"],
                                  ["--bytes-in-flight-kib", "48"]])
def test_memory_paths_usage_errors(args):
    r = run("b200gemm.cli.memory_paths", *args)
    assert r.returncode == 2 and r.stdout == ""


def test_memory_paths_needs_gpu_and_fails_cleanly():
    r = run("b200gemm.cli.memory_paths", "--stages", "4", "--bytes-in-flight-kib", "64",
            "--run-kind", "smoke")
    assert r.returncode == 1 and r.stdout == "" and "ERROR" in r.stderr


@pytest.mark.parametrize("args", [["--n", "96"], ["--depth", "5"], ["--iterations", "0"]])
def test_umma_usage_errors(args):
    r = run("b200gemm.cli.umma", *args)
    assert r.returncode == 2 and r.stdout == ""


def test_memory_paths_grids():
    sys.path.insert(0, ENV_PATH)
    from b200gemm.cli import memory_paths as mp
    ref = mp.reference_grid()
    assert len(ref) == 18 and {g[1] for g in ref} == {2, 4, 8}
    assert sorted({g[2] * g[1] // 1024 for g in ref}) == [16, 32, 64]
    base = mp.baseline_grid()
    assert {g[3] for g in base} == {1, 2, 4} and {g[2] for g in base} == {16384}


FAKE_NCU_CSV = '''==PROF== Connected to process
"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"
"0","1","python","h","ldgsts_stream_kernel","1","7","(128, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","dram__bytes_read.sum","byte","1,073,825,792"
"0","1","python","h","ldgsts_stream_kernel","1","7","(128, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","us","157.70"
"0","1","python","h","ldgsts_stream_kernel","1","7","(128, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","sm__cycles_elapsed.avg.per_second","Ghz","1.50"
'''


def test_ncu_bridge_parsing_and_classification():
    sys.path.insert(0, ENV_PATH)
    from b200gemm.cli import ncu_bridge as nb
    m = nb.parse_csv(FAKE_NCU_CSV)
    assert m["dram__bytes_read.sum"] == 1073825792
    assert abs(m["gpu__time_duration.sum"] - 157.7e-6) < 1e-12
    r = nb.summarise("memory", m, useful_bytes=1 << 30)
    assert r["classification"] == "HBM_VALIDATED" and r["flags"] == []
    assert abs(r["effective_gbps"] - (1 << 30) / 157.7e-6 / 1e9) < 1e-6
    r = nb.summarise("memory", m, useful_bytes=(1 << 30) * 2)
    assert r["classification"] == "INCONCLUSIVE"
    t = nb.summarise("tensor", m, flop=2 * 8192 ** 3)
    assert abs(t["sm_clock_ghz"] - 1.5) < 1e-9
    cmd = nb.ncu_command("memory", "ldgsts", 1, ["python", "x.py"])
    assert cmd[:3] == ["ncu", "--clock-control", "none"] and "--launch-count" in cmd


def test_ncu_bridge_usage():
    assert run("b200gemm.cli.ncu_bridge", "--kind", "memory").returncode == 2
    r = run("b200gemm.cli.ncu_bridge", "--kind", "memory", "--kernel", "x", "--", "true")
    assert r.returncode == 2  # memory kind needs --useful-bytes


def test_schedule_options_parse():
    from b200gemm.cli import gemm_comparison
    p = gemm_comparison.build_arg_parser()
    assert p.parse_args([]).schedule == "auto"
    assert p.parse_args(["--schedule", "streamk"]).schedule == "streamk"
    r = subprocess.run([sys.executable, str(REPO / "bench.py"), "--schedule", "sometimes"],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 2 and "--schedule" in r.stderr


def test_row_contracts_match_the_reference_headers():
    """The drivers' reference schemas are the reference's own headers, column for
    column (fixture extracted from its sources by tests/golden/make_golden.py)."""
    import json
    sys.path.insert(0, ENV_PATH)
    from b200gemm.cli import gemm_comparison as gc, memory_paths as mp, row_contracts as rc, umma
    g = json.loads((REPO / "tests" / "golden" / "row_contracts.json").read_text())
    assert list(rc.P35_FIELDS) == g["p35"] and len(rc.P35_FIELDS) == 100
    assert list(rc.MEM_FIELDS) == g["memory"]["ldgsts"] == g["memory"]["tma"]
    assert list(rc.UMMA_FIELDS) == g["umma"]["umma_1sm"] == g["umma"]["umma_2sm"]
    # The default b200 schemas keep the reference columns first, in order.
    assert gc.CSV_FIELDS[:100] == rc.P35_FIELDS
    assert mp.CSV_FIELDS[:37] == rc.MEM_FIELDS
    assert umma.CSV_FIELDS[:37] == rc.UMMA_FIELDS
    assert set(rc.KERNEL_ONLY_FIELDS) <= set(rc.P35_FIELDS)
    assert set(rc.CUBLASLT_ONLY_FIELDS) <= set(rc.P35_FIELDS)


def test_p35_value_conventions():
    sys.path.insert(0, ENV_PATH)
    from b200gemm.cli import row_contracts as rc
    t = rc.p35_text({"kernel_time_ms": 0.5190001, "tflops": 2118.5, "max_abs_error": 0.0,
                     "gap_to_cublaslt_pct": -12.5, "use_2cta_instrs": True, "m": 8192,
                     "throughput_ratio_vs_cublaslt": 1.25, "atol": 0.1})
    assert t["kernel_time_ms"] == "0.519000" and t["tflops"] == "2118.500000"
    assert t["max_abs_error"] == "0.000000000" and t["gap_to_cublaslt_pct"] == "-12.500000"
    assert t["use_2cta_instrs"] == "true" and t["m"] == "8192" and t["atol"] == "0.100000000"
    assert t["throughput_ratio_vs_cublaslt"] == "1.250000000"
    assert t["algo_id"] == "not_applicable" and len(t) == 100
