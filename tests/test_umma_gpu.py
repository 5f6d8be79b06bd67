"""UMMA probe: exact known answer (integer pattern) and seeded bf16 within tolerance.

Exact: D == depth * A * B^T for the reference's integer pattern, every
(cta_group, N, depth) of the union grid {64,128,256} x {4,16,32,64,128,256}.
Seeded uniform[-1,1) inputs: |D - depth*A*B^T| <= depth * 16 * 2^-22 * (1 + |R|)
(fp32 accumulation of `depth` identical partial products).
"""
import numpy as np
import pytest
import torch

from b200gemm import umma
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cta_group", [1, 2])
@pytest.mark.parametrize("n", [64, 128, 256])
@pytest.mark.parametrize("depth", [4, 16, 32, 64, 128, 256])
def test_integer_pattern_exact(cta_group, n, depth):
    d, cycles, status = umma.run_probe(cta_group, n, depth, iterations=2, timed=True)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = oracle.umma_reference(cta_group, n, depth)
    assert np.array_equal(d.cpu().double().numpy(), ref)
    assert int(cycles[0].item()) > 0


@pytest.mark.parametrize("cta_group", [1, 2])
def test_seeded_uniform(cta_group):
    g = torch.Generator().manual_seed(0)
    m, n, depth = 128 * cta_group, 256, 64
    a = (torch.rand((m, 16), generator=g) * 2 - 1).to(torch.bfloat16)
    b = (torch.rand((n, 16), generator=g) * 2 - 1).to(torch.bfloat16)
    d, _, status = umma.run_probe(cta_group, n, depth, iterations=3, a=a, b=b)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = depth * oracle.gemm_tn_f64(a, b)
    err = np.abs(d.cpu().double().numpy() - ref)
    assert float(err.max()) <= depth * 16 * 2 ** -22 * (1 + np.abs(ref).max())


def test_many_ctas_all_sms():
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    d, cycles, status = umma.run_probe(1, 256, 256, iterations=50, timed=True, num_ctas=sms)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert bool((cycles > 0).all())
    assert np.array_equal(d.cpu().double().numpy(), oracle.umma_reference(1, 256, 256))
