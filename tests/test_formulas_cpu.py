"""Reported-metric arithmetic and result checks against the reference's own outputs
(tests/golden/formulas.json and validate.json were produced by running the
reference's gemm_comparison.py and analyze_exp01_memory_paths_p14.py)."""
import json

import pytest
import torch

from b200gemm import check, formulas
from b200gemm._lib import CorrectnessError


def test_flop_and_tflops(golden_dir):
    g = json.loads((golden_dir / "formulas.json").read_text())
    for row in g["flop"]:
        m, n, k, _ = row["shape"]
        assert formulas.compute_flop_count(m, n, k) == row["flop_count"]
    for row in g["tflops"]:
        assert formulas.compute_tflops(row["flop_count"], row["ms"]) == pytest.approx(
            row["tflops"], rel=1e-15)


def test_ratio_gap(golden_dir):
    g = json.loads((golden_dir / "formulas.json").read_text())
    for case in g["comparison"]:
        m, n, k, _ = case["shape"]
        flop = formulas.compute_flop_count(m, n, k)
        base = formulas.compute_tflops(flop, case["times"][3])
        for t, row in zip(case["times"], case["rows"]):
            tf = formulas.compute_tflops(flop, t)
            assert tf == pytest.approx(row["tflops"], rel=1e-15)
            ratio, gap = formulas.compute_ratio_and_gap(tf, base)
            assert ratio == pytest.approx(row["throughput_ratio_vs_cublaslt"], rel=1e-12)
            assert gap == pytest.approx(row["gap_to_cublaslt_pct"], abs=1e-9)


def test_classify_hbm(golden_dir):
    g = json.loads((golden_dir / "formulas.json").read_text())
    for case in g["classify_hbm"]:
        got = formulas.classify_hbm(case["dram"], case["useful"])
        assert [got[0], got[1], got[2]] == case["result"]


def test_validate_result_matches_reference(golden_dir):
    g = json.loads((golden_dir / "validate.json").read_text())
    ref = torch.tensor(g["reference"]).reshape(g["shape"])
    for name, case in g["cases"].items():
        res = torch.tensor(case["result"]).reshape(g["shape"])
        if case["ok"]:
            max_abs, max_rel = check.validate_result(name, ref, res)
            assert max_abs == pytest.approx(case["max_abs"], abs=0)
            assert max_rel == pytest.approx(case["max_rel"], abs=0)
        else:
            with pytest.raises(CorrectnessError):
                check.validate_result(name, ref, res)


def test_validate_result_rejects_nan():
    ref = torch.zeros(4, 4)
    res = torch.zeros(4, 4)
    res[1, 1] = float("nan")
    with pytest.raises(CorrectnessError):
        check.validate_result("nan", ref, res)


def test_bf16_tolerance():
    g = torch.Generator().manual_seed(0)
    ref = torch.randn(64, 64, generator=g, dtype=torch.float64) * 30
    res = ref.to(torch.bfloat16)
    stats = check.bf16_tolerance_check("rounded", ref, res, 64, 1.0, 1.0)
    assert stats["violations"] == 0
    bad = res.clone()
    bad[0, 0] = bad[0, 0] * 1.1 + 1
    with pytest.raises(CorrectnessError):
        check.bf16_tolerance_check("bad", ref, bad, 64, 1.0, 1.0)


def test_umma_and_stream_formulas():
    assert formulas.umma_flop_count(128, 256, 256, 1000) == 2 * 128 * 256 * 16 * 256 * 1000
    assert formulas.effective_gbps(10 ** 9, 1000.0) == pytest.approx(1.0)
    assert formulas.flops_per_cycle_per_sm(8192 * 100, 100, 1) == 8192
    with pytest.raises(formulas.FormulaError):
        formulas.compute_tflops(10, 0.0)
