"""The allocation-free GEMM entry point, b200_gemm_noalloc, on the GPU.

Some callers cannot allocate device memory (they give all of it to their own
pool up front, or must not take the device-wide synchronisation that
cudaMalloc/cudaFree imply). b200_gemm_noalloc serves them: it keeps the
kernel's only scratch -- its status word and tile counter -- in a static device array of the
library. This test calls it through the C ABI twice in a row, on different
operands, and checks each result against the existing entry point b200_gemm
(bit-identical: same kernel) and against the CPU oracle with the bf16
tolerance the other GEMM tests use. It runs last (file name), and also passes
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
    rc = fn(m, n, k, a.data_ptr(), b.data_ptr(), d.data_ptr(), n, _lib.OUT_BF16, mode, stream)
    assert rc == _lib.OK, _lib.last_error()


@pytest.mark.parametrize("mode", [_lib.MODE_2CTA, _lib.MODE_1CTA])
def test_noalloc_matches_existing_entry_point(mode):
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call, (m, n, k, seed) in enumerate([(512, 768, 320, 21), (384, 256, 1024, 22)]):
        a, b = operands.uniform_operands(m, n, k, seed=seed)
        a_d, b_d = a.to(dev), b.to(dev)
        d_existing = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=dev)
        d_noalloc = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=dev)
        _call(lib.b200_gemm, a_d, b_d, d_existing, mode, stream)
        _call(lib.b200_gemm_noalloc, a_d, b_d, d_noalloc, mode, stream)
        torch.cuda.synchronize()
        got, want = d_noalloc.cpu(), d_existing.cpu()
        assert torch.equal(got, want), f"call {call}: differs from b200_gemm"
        ref = torch.from_numpy(oracle.gemm_tn_f64(a, b))
        check.bf16_tolerance_check(f"noalloc call {call}", ref, got, k, 1.0, 1.0)


def test_noalloc_rejects_bad_arguments():
    lib = _lib.load()
    rc = lib.b200_gemm_noalloc(64, 64, 60, 16, 16, 16, 64, _lib.OUT_BF16, 0, None)
    assert rc == _lib.ERR_UNSUPPORTED and "K" in _lib.last_error()
    rc = lib.b200_gemm_noalloc(64, 64, 64, None, None, None, 64, _lib.OUT_BF16, 0, None)
    assert rc == _lib.ERR_INVALID_ARGUMENT
