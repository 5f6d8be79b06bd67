"""GEMM parity on the GPU through the C ABI, against the CPU oracle and golden fixtures.

Tolerances (written here, used below):
  bf16 output: rel. Frobenius <= 1e-2 and per element
               |D - R| <= ulp_bf16(|R| + eps)/2 + eps, eps = 2^-20 * K * max|a| * max|b|
  fp32 output: the reference's rule |D - R| <= 1e-1 + 1e-5 |R| (gemm_comparison.py:152-154)
  integer operands (reference's factory): exact, max_abs_error == 0
"""
import json

import numpy as np
import pytest
import torch

from b200gemm import check, gemm as G, operands
from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def run(a, b, out_dtype=torch.bfloat16, mode="auto"):
    a_d, b_d = a.to(DEV), b.to(DEV)
    out = torch.full((a.shape[0], b.shape[0]), float("nan"), dtype=out_dtype, device=DEV)
    G.gemm(a_d, b_d, out, mode=mode)
    return out.cpu()


def maxabs(t):
    return float(t.float().abs().max()) if t.numel() else 0.0


@pytest.mark.parametrize("mode", ["1cta", "2cta", "2cta_m512", "2cta_n128"])
@pytest.mark.parametrize("shape", [(128, 256, 64), (96, 80, 72), (200, 264, 136), (256, 512, 256)])
def test_small_golden(golden_dir, shape, mode):
    z = np.load(golden_dir / "gemm_small.npz")
    tag = "x".join(map(str, shape))
    a = torch.from_numpy(z[f"a_{tag}"]).view(torch.bfloat16)
    b = torch.from_numpy(z[f"b_{tag}"]).view(torch.bfloat16)
    ref = torch.from_numpy(z[f"d_{tag}"])
    d = run(a, b, torch.bfloat16, mode)
    check.bf16_tolerance_check(f"{tag}/{mode}", ref, d, shape[2], maxabs(a), maxabs(b))
    d32 = run(a, b, torch.float32, mode)
    check.validate_result(f"{tag}/{mode}/f32", ref, d32)
    # fp32 output against the double oracle: only accumulation-order error.
    ref64 = torch.from_numpy(oracle.gemm_tn_f64(a, b))
    assert float((d32.double() - ref64).abs().max()) <= 2.0 ** -20 * shape[2]


@pytest.mark.parametrize("mode", ["1cta", "2cta", "2cta_m512", "2cta_n128", "auto"])
def test_c1_512(golden_dir, mode):
    g = json.loads((golden_dir / "gemm_512.json").read_text())
    a, b = operands.uniform_operands(512, 512, 512, seed=0)
    import hashlib
    assert hashlib.sha256(a.view(torch.int16).numpy().tobytes()).hexdigest() == g["a_sha256"]
    assert hashlib.sha256(b.view(torch.int16).numpy().tobytes()).hexdigest() == g["b_sha256"]
    d = run(a, b, torch.bfloat16, mode)
    ref = torch.from_numpy(oracle.gemm_tn_f64(a, b))
    check.bf16_tolerance_check(f"512/{mode}", ref, d, 512, maxabs(a), maxabs(b))
    idx = np.array(g["idx"])
    sampled = d.double().numpy()[idx[:, 0], idx[:, 1]]
    assert np.allclose(sampled, np.array(g["values"]), rtol=2 ** -7, atol=2 ** -10 * 512)


@pytest.mark.parametrize("shape", [(1, 8, 8), (17, 24, 8), (129, 264, 72), (300, 1000, 520),
                                   (640, 136, 4104), (1000, 16, 64), (1100, 520, 200),
                                   (384, 104, 256), (384, 128, 64), (2048, 64, 512)])
@pytest.mark.parametrize("mode", ["1cta", "2cta", "2cta_m512", "2cta_n128"])
def test_ragged_shapes(shape, mode):
    m, n, k = shape
    a, b = operands.uniform_operands(m, n, k, seed=3)
    d = run(a, b, torch.bfloat16, mode)
    ref = torch.from_numpy(oracle.gemm_tn_f64(a, b))
    check.bf16_tolerance_check(f"{shape}/{mode}", ref, d, k, maxabs(a), maxabs(b))


def test_strided_output_placement():
    """D written at a column offset inside a wider matrix (ldd > N), neighbours untouched."""
    m, n, k, ld = 256, 256, 128, 1024
    a, b = operands.uniform_operands(m, n, k, seed=4)
    big = torch.full((m, ld), -7.0, dtype=torch.bfloat16, device=DEV)
    view = big[:, 256:512]
    G.gemm(a.to(DEV), b.to(DEV), view)
    host = big.cpu()
    ref = torch.from_numpy(oracle.gemm_tn_f64(a, b))
    check.bf16_tolerance_check("strided", ref, host[:, 256:512], k, maxabs(a), maxabs(b))
    assert bool((host[:, :256] == -7.0).all()) and bool((host[:, 512:] == -7.0).all())


def test_ref_compat_exact(golden_dir):
    """The reference's integer operands (cutlass factory, seed 1111): fp32 D is exact."""
    z = np.load(golden_dir / "ref_small.npz")
    a = torch.from_numpy(z["a"]).view(torch.bfloat16)
    b = torch.from_numpy(z["b"]).view(torch.bfloat16)
    ref = torch.from_numpy(z["d"])
    for mode in ("1cta", "2cta", "2cta_m512", "2cta_n128"):
        d = run(a, b, torch.float32, mode)
        max_abs, _ = check.validate_result("ref_compat", ref, d)
        assert max_abs == 0.0


def test_reference_bridge_signature():
    """b200_gemm_plan_create keeps p35_plan_create's argument list and fp32 D contract."""
    m, n, k = 256, 512, 128
    a, b = operands.integer_operands(m, n, k)
    a_d, b_d = a.to(DEV), b.to(DEV)
    d = torch.full((m, n), float("nan"), dtype=torch.float32, device=DEV)
    br = G.B200GemmBridge()
    info = br.create_plan(m, n, k, a_d.data_ptr(), b_d.data_ptr(), d.data_ptr(), d.data_ptr(),
                          torch.cuda.current_stream().cuda_stream)
    assert info.m == m and info.out_dtype == 1
    br.execute()
    br.synchronize()
    br.destroy()
    ref = a.float() @ b.float().T
    assert torch.equal(d.cpu(), ref)


def test_plan_reuse_and_repeat():
    m, n, k = 512, 768, 512
    a, b = operands.uniform_operands(m, n, k, seed=5)
    a_d, b_d = a.to(DEV), b.to(DEV)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=DEV)
    plan = G.GemmPlan(a_d, b_d, out, mode="2cta_m512")
    plan.execute()
    plan.synchronize()
    first = out.clone()
    for _ in range(5):
        out.fill_(float("nan"))
        plan.execute()
    plan.synchronize()
    plan.destroy()
    assert torch.equal(first, out)  # deterministic, no race between tiles


def test_empty_and_invalid():
    a = torch.empty((0, 64), dtype=torch.bfloat16, device=DEV)
    b = torch.empty((32, 64), dtype=torch.bfloat16, device=DEV)
    out = G.gemm(a, b)
    assert out.shape == (0, 32)
    ok, why = G.supported(64, 64, 60)
    assert not ok and "K" in why
    with pytest.raises(G.BridgeError):
        x = torch.zeros((64, 60), dtype=torch.bfloat16, device=DEV)
        G.gemm(x, x)


def test_unaligned_pitch_rejected():
    """A D row pitch that is not a multiple of 16 bytes is refused with a clear error."""
    ok, why = G.supported(64, 257, 64)
    assert not ok and "16 bytes" in why
    ok, _ = G.supported(64, 257, 64, out_dtype=torch.float32, ldd=260)
    assert ok


@pytest.mark.parametrize("mode", ["1cta", "2cta", "2cta_m512", "2cta_n128"])
@pytest.mark.parametrize("n", [16, 64, 104, 128, 192])
def test_narrow_n_strided_repeat(mode, n):
    """Output narrower than one 256-column tile (some 64-column chunks fall
    outside D), placed in a wider zeroed buffer, five launches in a row: every
    element of D is written every time and nothing outside it."""
    m, k, ld = 384, 256, 256
    a, b = operands.uniform_operands(m, n, k, seed=6)
    ref = torch.from_numpy(oracle.gemm_tn_f64(a, b))
    for _ in range(5):
        big = torch.zeros((m, ld), dtype=torch.bfloat16, device=DEV)
        G.gemm(a.to(DEV), b.to(DEV), big[:, :n], mode=mode)
        host = big.cpu()
        check.bf16_tolerance_check(f"narrow {n}/{mode}", ref, host[:, :n], k, maxabs(a), maxabs(b))
        assert bool((host[:, n:] == 0).all())


@pytest.mark.parametrize("mode", ["1cta", "2cta", "2cta_m512", "2cta_n128"])
def test_launch_after_producer_kernel_sees_its_writes(mode):
    """Plans launch with programmatic dependent launch: a GEMM that follows a
    kernel writing its operand must still read the new values (no global access
    before griddepcontrol.wait), launch after launch on one stream."""
    m, n, k = 1024, 768, 512
    a, b = operands.uniform_operands(m, n, k, seed=7)
    a_d, b_d = a.to(DEV), b.to(DEV)
    outs = [torch.empty((m, n), dtype=torch.float32, device=DEV) for _ in range(6)]
    plans = [G.GemmPlan(a_d, b_d, o, mode=mode) for o in outs]
    for i, plan in enumerate(plans):
        a_d.mul_(-1.0 if i % 2 == 0 else 2.0)  # an elementwise kernel right before the GEMM
        plan.execute()
    for plan in plans:
        plan.synchronize()
        plan.destroy()
    ref = a.double() @ b.double().T
    scale = 1.0
    for i, o in enumerate(outs):
        scale *= -1.0 if i % 2 == 0 else 2.0
        err = float((o.cpu().double() - scale * ref).abs().max())
        assert err <= 1e-2 * abs(scale), (i, err)
