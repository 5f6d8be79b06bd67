"""Full-size checks at the benchmark configurations' real sizes.

GEMM: against torch's IEEE fp32 matmul on the GPU (the reference's own oracle,
src/gemm/gemm_comparison.py:2705-2722) on sampled rows, with the bf16 tolerance
of the other GEMM tests; plus size-independent exact properties: scaling A by 2
scales D by exactly 2 (powers of two are exact in bf16 and fp32), and permuting
the rows of A inside their 128-row blocks permutes the rows of D bit for bit
(a row's dot products depend only on the tiles that hold it, not on its
position among them).
Streams: the 4 GiB seeded bf16 buffer of the memory-path config, checksummed
by LDGSTS and TMA, equal bit for bit to the host's checksum of the same bytes.
"""
import numpy as np
import pytest
import torch

from b200gemm import check, gemm as G, memory_paths as mp, operands

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


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


def sampled_check(a, b, out, rows, label):
    torch.backends.cuda.matmul.allow_tf32 = False
    ref = a[rows].float() @ b.float().T
    k = a.shape[1]
    check.bf16_tolerance_check(label, ref.cpu(), out[rows].cpu(), k,
                               float(a.float().abs().max()), float(b.float().abs().max()))


@pytest.mark.parametrize("shape,kind", [((8192, 8192, 8192), "square"),
                                        ((16384, 16384, 16384), "square"),
                                        ((8192, 128256, 4096), "llm")])
def test_full_size_sampled_rows(shape, kind):
    m, n, k = shape
    if kind == "square":
        a, b = operands.square_operands(m, seed=1)
    else:
        a, b = operands.llm_operands(n, k, m=m)
    a, b = a.to(DEV), b.to(DEV)
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=DEV)
    G.gemm(a, b, out)  # AUTO mode, as bench.py and the drivers use it
    assert not bool(torch.isnan(out).any())
    rows = torch.randint(0, m, (128,), generator=torch.Generator().manual_seed(0)).to(DEV)
    sampled_check(a, b, out, rows, f"{shape}")


@pytest.mark.parametrize("mode", ["2cta", "2cta_m512"])
def test_exact_properties_8192(mode):
    m = n = k = 8192
    a, b = operands.square_operands(m, seed=1)
    a, b = a.to(DEV), b.to(DEV)
    d1 = torch.empty((m, n), dtype=torch.float32, device=DEV)
    d2 = torch.empty_like(d1)
    G.gemm(a, b, d1, mode=mode)
    G.gemm(a * 2, b, d2, mode=mode)
    assert torch.equal(d2, d1 * 2)
    perm = block_perm(m, 128, seed=1).to(DEV)
    d3 = torch.empty_like(d1)
    G.gemm(a[perm].contiguous(), b, d3, mode=mode)
    assert torch.equal(d3, d1[perm])


def test_stream_4gib_checksum_bit_exact():
    nbytes = 4 << 30
    g = torch.Generator(device=DEV).manual_seed(2)
    buf = torch.empty(nbytes // 2, dtype=torch.bfloat16, device=DEV)
    chunk = 1 << 28
    for i in range(0, buf.numel(), chunk):  # seeded uniform[-1, 1) bf16, 4 GiB
        buf[i:i + chunk] = (torch.rand(min(chunk, buf.numel() - i), generator=g, device=DEV) * 2 - 1)
    words = buf.view(torch.int32).cpu().numpy().view(np.uint32)
    host = (int(np.bitwise_xor.reduce(words)), int(words.sum(dtype=np.uint64)))
    del words
    for method, stages, sb, ctas in (("ldgsts", 4, 16384, 2), ("tma_sw128", 2, 16384, 4),
                                     ("tma", 4, 16384, 1)):
        assert mp.device_checksum(buf, method, stages=stages, stage_bytes=sb, ctas_per_sm=ctas) == host
