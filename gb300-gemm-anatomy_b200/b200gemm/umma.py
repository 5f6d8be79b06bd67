"""UMMA throughput probe front end (tcgen05.mma kind::f16, operands in SMEM).

Replaces the reference's umma_1sm / umma_2sm binaries
(src/compute/umma_1sm.cu:1020-1060 run_once, src/compute/umma_2sm.cu). The
known answer of the integer pattern is D = depth * A * B^T with
A[r,k] = ((r+3k) mod 7) - 3 and B[k,c] = ((2k+c) mod 5) - 2
(umma_1sm.cu:577-586; global rows/cols in 2-CTA mode, umma_2sm.cu:513-527).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

N_VALUES = (64, 128, 256)
DEPTHS = (4, 16, 32, 64, 128, 256)
REF_DEPTHS = (4, 16, 64, 256)


def run_probe(cta_group: int, n: int, depth: int, iterations: int = 1, timed: bool = False,
              a: torch.Tensor | None = None, b: torch.Tensor | None = None, num_ctas: int = 0,
              device: int = 0, stream=None):
    """Launch the probe; returns (D [M x N] fp32 on device, cycles [ctas] uint64 on device, status)."""
    lib = _lib.load()
    dev = torch.device("cuda", device)
    m = 128 * cta_group
    d = torch.full((m, n), float("nan"), dtype=torch.float32, device=dev)
    ctas = max(num_ctas, 1) * cta_group
    cycles = torch.zeros(ctas, dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    if (a is None) != (b is None):
        raise ValueError("pass both a and b, or neither (integer pattern)")
    if a is not None:
        if a.shape != (m, 16) or b.shape != (n, 16) or a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
            raise ValueError(f"a must be bf16 {m}x16 and b bf16 {n}x16")
        a = a.to(dev).contiguous()
        b = b.to(dev).contiguous()
    cfg = _lib.UmmaConfig(cta_group, n, depth, iterations, 1 if timed else 0, num_ctas)
    s = torch.cuda.current_stream(dev) if stream is None else stream
    rc = lib.b200_umma_probe(ctypes.byref(cfg), a.data_ptr() if a is not None else None,
                             b.data_ptr() if b is not None else None, d.data_ptr(),
                             cycles.data_ptr(), status.data_ptr(), int(s.cuda_stream))
    _lib.check(rc, "b200_umma_probe", lib)
    return d, cycles, status
