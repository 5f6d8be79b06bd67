"""The allocation-free GEMM entry point, b200_gemm_noalloc, on the GPU.

Some callers cannot allocate device memory (they give all of it to their own
pool up front, or must not take the device-wide synchronisation that
cudaMalloc/cudaFree imply). b200_gemm_noalloc serves them: it keeps the
kernel's only scratch -- its status word and tile counter -- in a static device array of the
library. This test calls it through the C ABI twice in a row, on different
operands, in every mode and for both output types, and checks each result
against the existing entry point b200_gemm (bit-identical: same kernel, grid
and schedule at these sizes) and against the CPU oracle with the tolerance the
other GEMM tests use; it also checks that a call leaves free device memory
unchanged, and a 4096^3 call, where b200_gemm would take the stream-K schedule
and this entry point keeps the dynamic one. It runs last (file name), and also passes
alone in a fresh process.
"""
import ctypes

import pytest
import torch

from b200gemm import _lib, check, operands
from oracle import oracle

pytestmark = pytest.mark.gpu


def _call(fn, a, b, d, mode, stream):
    m, k = a.shape
    n = b.shape[0]
    out_dtype = _lib.OUT_F32 if d.dtype == torch.float32 else _lib.OUT_BF16
    rc = fn(m, n, k, a.data_ptr(), b.data_ptr(), d.data_ptr(), n, out_dtype, mode, stream)
    assert rc == _lib.OK, _lib.last_error()


@pytest.mark.parametrize("mode", [_lib.MODE_2CTA, _lib.MODE_1CTA, _lib.MODE_2CTA_M512,
                                  _lib.MODE_2CTA_N128, _lib.MODE_AUTO])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_existing_entry_point(mode, out_dtype):
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call, (m, n, k, seed) in enumerate([(1024, 768, 320, 21), (384, 256, 1024, 22)]):
        a, b = operands.uniform_operands(m, n, k, seed=seed)
        a_d, b_d = a.to(dev), b.to(dev)
        d_existing = torch.full((m, n), float("nan"), dtype=out_dtype, device=dev)
        d_noalloc = torch.full((m, n), float("nan"), dtype=out_dtype, device=dev)
        _call(lib.b200_gemm, a_d, b_d, d_existing, mode, stream)
        _call(lib.b200_gemm_noalloc, a_d, b_d, d_noalloc, mode, stream)
        torch.cuda.synchronize()
        got, want = d_noalloc.cpu(), d_existing.cpu()
        assert torch.equal(got, want), f"call {call}: differs from b200_gemm"
        ref = torch.from_numpy(oracle.gemm_tn_f64(a, b))
        if out_dtype == torch.bfloat16:
            check.bf16_tolerance_check(f"noalloc call {call}", ref, got, k, 1.0, 1.0)
        else:
            assert float((got.double() - ref).abs().max()) <= 2.0 ** -20 * k


def test_noalloc_allocates_nothing():
    """Free device memory is the same before and after a warmed-up call."""
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    a, b = operands.uniform_operands(2048, 2048, 512, seed=23)
    a_d, b_d = a.to(dev), b.to(dev)
    d = torch.empty((2048, 2048), dtype=torch.bfloat16, device=dev)
    _call(lib.b200_gemm_noalloc, a_d, b_d, d, _lib.MODE_AUTO, stream)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(dev)[0]
    for _ in range(3):
        _call(lib.b200_gemm_noalloc, a_d, b_d, d, _lib.MODE_AUTO, stream)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(dev)[0] == free0


def test_noalloc_on_a_stream_k_shape():
    """4096^3: b200_gemm takes the stream-K schedule there, the allocation-free
    entry point the dynamic one. Integer operands: both exact, so bit-identical;
    seeded uniform operands: within the bf16 rule of a float64 product."""
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    n = 4096
    a, b = operands.integer_operands(n, n, n, seed=24)
    a_d, b_d = a.to(dev), b.to(dev)
    d_existing = torch.full((n, n), float("nan"), dtype=torch.float32, device=dev)
    d_noalloc = torch.full((n, n), float("nan"), dtype=torch.float32, device=dev)
    _call(lib.b200_gemm, a_d, b_d, d_existing, _lib.MODE_AUTO, stream)
    _call(lib.b200_gemm_noalloc, a_d, b_d, d_noalloc, _lib.MODE_AUTO, stream)
    exact = a_d.double() @ b_d.double().T
    assert torch.equal(d_noalloc.double(), exact)
    assert torch.equal(d_existing, d_noalloc)
    a, b = operands.uniform_operands(n, n, n, seed=25)
    a_d, b_d = a.to(dev), b.to(dev)
    d = torch.full((n, n), float("nan"), dtype=torch.bfloat16, device=dev)
    _call(lib.b200_gemm_noalloc, a_d, b_d, d, _lib.MODE_AUTO, stream)
    ref = a_d.double() @ b_d.double().T
    rows = torch.arange(0, n, 37, device=dev)
    check.bf16_tolerance_check("noalloc 4096^3", ref[rows].cpu(), d[rows].cpu(), n, 1.0, 1.0)


def test_noalloc_rejects_bad_arguments():
    lib = _lib.load()
    rc = lib.b200_gemm_noalloc(64, 64, 60, 16, 16, 16, 64, _lib.OUT_BF16, 0, None)
    assert rc == _lib.ERR_UNSUPPORTED and "K" in _lib.last_error()
    rc = lib.b200_gemm_noalloc(64, 64, 64, None, None, None, 64, _lib.OUT_BF16, 0, None)
    assert rc == _lib.ERR_INVALID_ARGUMENT
