"""Failure detection on the GPU without faulting it.

A kernel waits on an mbarrier that nothing arrives on; its bounded wait must
give up within the budget, report B200_DEV_TIMEOUT_SELFTEST through the status
word, and leave the context usable (a GEMM right after still succeeds).
"""
import time

import pytest
import torch

from b200gemm import _lib, gemm as G, operands

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    t0 = time.perf_counter()
    rc = lib.b200_selftest_bounded_wait(20_000_000, status.data_ptr(),
                                        torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.OK, _lib.last_error()
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(status.item()) == 0x107
    assert elapsed < 5.0
    a, b = operands.uniform_operands(256, 256, 128, seed=1)
    out = G.gemm(a.to(dev), b.to(dev))
    ref = a.float() @ b.float().T
    assert float((out.cpu().float() - ref).abs().max()) < 0.1


def test_bounded_wait_argument_checks():
    lib = _lib.load()
    assert lib.b200_selftest_bounded_wait(0, 16, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.b200_selftest_bounded_wait(1000, None, None) == _lib.ERR_INVALID_ARGUMENT
