"""Generates the committed golden fixtures under tests/golden/ (run in the build container).

Each fixture comes from the reference's own code where that code can run on
a CPU, imported from a checkout of the reference repository:

  formulas.json      compute_flop_count / compute_tflops / compute_shape_comparison
                     (src/gemm/gemm_comparison.py:1626-1763) on fixed inputs;
                     classify_hbm (scripts/analyze_exp01_memory_paths_p14.py:1887-1903).
  validate.json      validate_result (gemm_comparison.py:2725-2762) on fixed CPU tensors.
  gemm_small.npz     seeded bf16 operands (uniform[-1,1), seed 0, A then B) and the
                     reference's oracle math (fp32 einsum "mkl,nkl->mnl",
                     gemm_comparison.py:2705-2722) evaluated on the CPU.
  gemm_512.json      the same for the 512^3 config: operand hashes and summary
                     statistics plus 4096 sampled entries of D.
  ref_operands.json  sha256 of the reference's operands for its five frozen shapes
                     (torch.manual_seed(1111) then cutlass.torch.matrix for A and B,
                     src/gemm/cublaslt_gemm.py:1568-1587) and for a small shape,
                     plus the small shape's fp32 einsum D (exact: integer operands).
  splitmix.json      SplitMix64 published value and the first pattern vectors.
  row_contracts.json the reference's CSV headers: CSV_FIELDS of
                     src/gemm/gemm_comparison.py (imported), and the header strings
                     printed by print_csv_header in src/memory/ldgsts.cu, src/memory/tma.cu,
                     src/compute/umma_1sm.cu and src/compute/umma_2sm.cu (read as text).

Usage: python tests/golden/make_golden.py /path/to/reference [row_contracts]
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "gb300-gemm-anatomy_b200"))
sys.path.insert(0, str(REPO))

from b200gemm import operands  # noqa: E402
from oracle import oracle  # noqa: E402


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.int16).numpy().tobytes()).hexdigest()


def _printed_header(source: Path) -> list:
    """The column names printed by a reference binary's print_csv_header()."""
    import re
    text = source.read_text()
    body = text[text.index("void print_csv_header()"):]
    body = body[: body.index("}")]
    literal = "".join(re.findall(r'"((?:[^"\\]|\\.)*)"', body))
    return literal.replace("\\n", "").strip().split(",")


def row_contracts(ref_root: Path) -> None:
    sys.path.insert(0, str(ref_root / "src" / "gemm"))
    import gemm_comparison as gc
    out = {"p35": list(gc.CSV_FIELDS),
           "memory": {n: _printed_header(ref_root / "src" / "memory" / f"{n}.cu")
                      for n in ("ldgsts", "tma")},
           "umma": {n: _printed_header(ref_root / "src" / "compute" / f"{n}.cu")
                    for n in ("umma_1sm", "umma_2sm")}}
    (HERE / "row_contracts.json").write_text(json.dumps(out, indent=1))


def main(ref_root: Path) -> None:
    sys.path.insert(0, str(ref_root / "src" / "gemm"))
    sys.path.insert(0, str(ref_root / "scripts"))
    import gemm_comparison as gc

    # ---------------------------------------------------------------- formulas
    shapes = [(4096, 4096, 4096, 1), (8192, 8192, 8192, 1), (16384, 512, 4096, 1),
              (32768, 512, 4096, 1), (512, 16384, 4096, 1), (512, 512, 512, 1)]
    times = [0.0785, 0.519, 0.1, 0.2, 0.05, 0.01]
    formulas = {"flop": [], "tflops": [], "comparison": []}
    for s, t in zip(shapes, times):
        f = gc.compute_flop_count(s)
        formulas["flop"].append({"shape": list(s), "flop_count": f})
        formulas["tflops"].append({"flop_count": f, "ms": t, "tflops": gc.compute_tflops(f, t)})
    cmp_in = [((8192, 8192, 8192, 1), [1.2, 0.9, 0.762, 0.519]),
              ((4096, 4096, 4096, 1), [0.15, 0.094, 0.0825, 0.0785])]
    for s, ts in cmp_in:
        formulas["comparison"].append({"shape": list(s), "times": ts,
                                       "rows": gc.compute_shape_comparison(s, ts)})
    try:
        import analyze_exp01_memory_paths_p14 as p14
        cases = [(1.0e9, 1.0e9), (0.5e9, 1.0e9), (1.2e9, 1.0e9), (0.95e9, 1.0e9), (None, 1.0e9)]
        formulas["classify_hbm"] = [
            {"dram": d, "useful": u, "result": list(p14.classify_hbm(d, u))} for d, u in cases]
    except Exception as exc:  # pragma: no cover - recorded, not fatal
        formulas["classify_hbm_error"] = repr(exc)
    (HERE / "formulas.json").write_text(json.dumps(formulas, indent=1))

    # ---------------------------------------------------------------- validate_result
    g = torch.Generator().manual_seed(7)
    ref = torch.randn(32, 48, 1, generator=g) * 100
    cases = {"exact": ref.clone(), "within": ref + 0.05, "outside": ref.clone()}
    cases["outside"][3, 5, 0] += 0.5
    val = {"reference": ref.flatten().tolist(), "shape": list(ref.shape), "cases": {}}
    for name, res in cases.items():
        try:
            out = gc.validate_result(torch, name, ref, res)
            val["cases"][name] = {"ok": True, "max_abs": out[0], "max_rel": out[1],
                                  "result": res.flatten().tolist()}
        except Exception as exc:
            val["cases"][name] = {"ok": False, "error": type(exc).__name__,
                                  "result": res.flatten().tolist()}
    (HERE / "validate.json").write_text(json.dumps(val))

    # ---------------------------------------------------------------- small GEMMs
    arrays = {}
    for (m, n, k) in [(128, 256, 64), (96, 80, 72), (200, 264, 136), (256, 512, 256)]:
        a, b = operands.uniform_operands(m, n, k, seed=0)
        d = oracle.reference_einsum(a, b)
        tag = f"{m}x{n}x{k}"
        arrays[f"a_{tag}"] = a.view(torch.int16).numpy()
        arrays[f"b_{tag}"] = b.view(torch.int16).numpy()
        arrays[f"d_{tag}"] = d.numpy()
    np.savez_compressed(HERE / "gemm_small.npz", **arrays)

    a, b = operands.uniform_operands(512, 512, 512, seed=0)
    d = oracle.reference_einsum(a, b).double()
    rng = np.random.default_rng(0)
    idx = rng.integers(0, 512, size=(4096, 2))
    (HERE / "gemm_512.json").write_text(json.dumps({
        "a_sha256": sha(a), "b_sha256": sha(b), "sum": float(d.sum()),
        "sumsq": float((d * d).sum()), "idx": idx.tolist(),
        "values": [float(d[i, j]) for i, j in idx]}))

    # ---------------------------------------------------------------- reference operands
    ref_ops = {"seed": operands.REF_SEED, "shapes": {}}
    for (m, n, k) in list(operands.REF_FROZEN_SHAPES) + [(256, 512, 128)]:
        a, b = operands.ref_compat_operands(m, n, k)
        ref_ops["shapes"][f"{m}x{n}x{k}"] = {"a_sha256": sha(a), "b_sha256": sha(b),
                                             "a_min": float(a.float().min()),
                                             "a_max": float(a.float().max())}
    a, b = operands.ref_compat_operands(256, 512, 128)
    np.savez_compressed(HERE / "ref_small.npz", a=a.view(torch.int16).numpy(),
                        b=b.view(torch.int16).numpy(), d=oracle.reference_einsum(a, b).numpy())
    (HERE / "ref_operands.json").write_text(json.dumps(ref_ops, indent=1))

    # ---------------------------------------------------------------- splitmix
    words = oracle.pattern_words(0, 64)
    (HERE / "splitmix.json").write_text(json.dumps({
        "seed0_first_output": oracle.SPLITMIX_SEED0_FIRST,
        "gamma": oracle.SPLITMIX_GAMMA,
        "pattern_words_0_64": words.tolist()}))
    row_contracts(ref_root)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    if len(sys.argv) not in (2, 3):
        sys.exit("usage: python tests/golden/make_golden.py /path/to/reference [row_contracts]")
    if len(sys.argv) == 3 and sys.argv[2] == "row_contracts":
        row_contracts(Path(sys.argv[1]))
    else:
        main(Path(sys.argv[1]))
