"""Full-size parity for every configuration whose AUTO route differs.

Each shape runs through the public plan API in AUTO mode, the way bench.py and
the drivers call it, so the tile shape and schedule under test are the ones a
user gets (pinned here against `b200_gemm_policy`):
  * bf16 D against torch's IEEE fp32 matmul on 128 sampled rows with the bf16
    rule of the other GEMM tests (the reference's own oracle,
    src/gemm/gemm_comparison.py:2705-2722);
  * fp32 D: scaling A by 2 scales D by exactly 2; two launches of one plan are
    bit-identical; permuting the rows of A inside their 128-row blocks (every
    tile height is a multiple of 128) permutes the rows of D bit for bit, under
    either schedule: a row's sums depend only on the tiles that hold it;
  * the reference's five frozen shapes with its integer operands (cutlass
    factory, seed 1111, fp32 D): max_abs_error == 0, the reference's published
    result (README.md:492-493).
"""
import hashlib
import json
from pathlib import Path

import pytest
import torch

from b200gemm import check, gemm as G, operands

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
GOLDEN = Path(__file__).resolve().parent / "golden"


def block_perm(m, block, seed):
    """A random permutation of the rows of A that keeps every row inside its
    aligned block of `block` rows. Each output row is then computed by the same
    tiles, which walk K in a direction fixed by the tile (the dynamic schedule
    runs odd waves from the last k-slice down), so D's rows permute bit for bit."""
    g = torch.Generator().manual_seed(seed)
    idx = torch.arange(m)
    for r0 in range(0, m, block):
        r1 = min(m, r0 + block)
        idx[r0:r1] = r0 + torch.randperm(r1 - r0, generator=g)
    return idx

# (M, N, K), expected (mode, schedule) on a 148-SM B200, why it is here.
AUTO_SHAPES = [
    ((4096, 4096, 4096), ("2cta", "stream_k")),      # c4 square, 3.46 waves
    ((32768, 512, 4096), ("2cta", "stream_k")),      # frozen skinny, lanes along N
    ((8192, 4096, 4096), ("2cta", "dynamic")),       # c5
    ((8192, 14336, 4096), ("2cta", "dynamic")),      # c5
    ((8192, 4096, 14336), ("2cta", "dynamic")),      # c5, long K
    ((8192, 1792, 4096), ("2cta", "stream_k")),      # 8-GPU shard of N = 14336
    ((8192, 16032, 4096), ("2cta_m512", "dynamic")), # 8-GPU shard of N = 128256
    ((8192, 512, 4096), ("2cta", "dynamic")),        # 8-GPU shard of N = 4096 (64 tiles)
]


def _operands(m, n, k):
    if m == n == k:
        a, b = operands.square_operands(m, seed=1)
        return a.to(DEV), b.to(DEV)
    return operands.llm_operands_device(n, k, DEV, m=m)


@pytest.mark.parametrize("shape,route", AUTO_SHAPES, ids=lambda v: "x".join(map(str, v))
                         if isinstance(v[0], int) else "-".join(v))
def test_auto_route_full_size(shape, route):
    m, n, k = shape
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    pol = G.policy(m, n, k, sm_count=sms)
    if sms == 148:
        assert (pol["mode"], pol["schedule"]) == route
    a, b = _operands(m, n, k)
    torch.backends.cuda.matmul.allow_tf32 = False
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=DEV)
    plan = G.GemmPlan(a, b, out)
    assert plan.schedule == pol["schedule"]
    plan.execute()
    plan.synchronize()
    plan.destroy()
    rows = torch.randint(0, m, (128,), generator=torch.Generator().manual_seed(3)).to(DEV)
    ref = a[rows].float() @ b.float().T
    check.bf16_tolerance_check(f"{shape} auto", ref.cpu(), out[rows].cpu(), k,
                               float(a.float().abs().max()), float(b.float().abs().max()))
    del out, ref

    d1 = torch.empty((m, n), dtype=torch.float32, device=DEV)
    p1 = G.GemmPlan(a, b, d1)
    p1.execute()
    p1.synchronize()
    first = d1.clone()
    p1.execute()
    p1.synchronize()
    p1.destroy()
    assert torch.equal(first, d1), "two launches of one plan differ"
    a2 = a * 2
    d2 = torch.empty_like(d1)
    G.gemm(a2, b, d2)
    assert torch.equal(d2, d1 * 2)
    del a2, d2
    perm = block_perm(m, 128, seed=1).to(DEV)
    d3 = torch.empty_like(d1)
    G.gemm(a[perm].contiguous(), b, d3)
    assert torch.equal(d3, d1[perm])


@pytest.mark.parametrize("shape", operands.REF_FROZEN_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_frozen_shapes_reference_operands_exact(shape):
    """AUTO mode, fp32 D, the reference's operands: every element exact."""
    m, n, k = shape
    if operands.ref_compat_available():
        a, b = operands.ref_compat_operands(m, n, k)
        pins = json.loads((GOLDEN / "ref_operands.json").read_text())["shapes"][f"{m}x{n}x{k}"]
        assert hashlib.sha256(a.view(torch.int16).numpy().tobytes()).hexdigest() == pins["a_sha256"]
        assert hashlib.sha256(b.view(torch.int16).numpy().tobytes()).hexdigest() == pins["b_sha256"]
    else:
        a, b = operands.integer_operands(m, n, k)
    a, b = a.to(DEV), b.to(DEV)
    d = torch.full((m, n), float("nan"), dtype=torch.float32, device=DEV)
    G.gemm(a, b, d)
    exact = a.double() @ b.double().T  # integer sums: exact in fp64 (and in fp32)
    max_abs, _ = check.validate_result(f"{shape} ref_compat auto", exact.float(), d)
    assert max_abs == 0.0
