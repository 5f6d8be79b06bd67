"""Seeded synthetic operands for every benchmark configuration.

All operands are drawn on the host with a seeded ``torch.Generator`` (A before
B, then cast to bf16), so the host copy the oracle sees is bit-identical to
what is uploaded. Configurations (names follow the benchmark configs):

  c1  M=N=K=512, uniform[-1,1), seed 0
  c4  square M=N=K in {4096, 8192, 16384}, N(0,1)*0.1, seed 1
  c5  M=8192 activations N(0,1), weights N(0,0.02), seed 2

``ref_compat`` reproduces the reference driver's operand path: seed 1111, then
the CUTLASS DSL factory ``cutlass.torch.matrix`` for A, then B
(src/gemm/cublaslt_gemm.py:1568-1587, gemm_comparison.py:2633-2666); on the
installed factory the values are small integers in {-2..1}, so every fp32 dot
product is exact and the reference's published max_abs_error is 0.
"""
from __future__ import annotations

import torch

SQUARE_SIZES = (4096, 8192, 16384)
LLM_M = 8192
LLM_NK = ((4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096))
REF_FROZEN_SHAPES = ((4096, 4096, 4096), (8192, 8192, 8192), (16384, 512, 4096),
                     (32768, 512, 4096), (512, 16384, 4096))
REF_SEED = 1111


def _uniform(g, shape, lo=-1.0, hi=1.0):
    return (torch.rand(shape, generator=g, dtype=torch.float32) * (hi - lo) + lo).to(torch.bfloat16)


def _normal(g, shape, std):
    return (torch.randn(shape, generator=g, dtype=torch.float32) * std).to(torch.bfloat16)


def uniform_operands(m: int, n: int, k: int, seed: int = 0):
    """A (M x K), B (N x K) bf16 ~ uniform[-1, 1) from `seed`, A drawn first (config c1)."""
    g = torch.Generator().manual_seed(seed)
    a = _uniform(g, (m, k))
    b = _uniform(g, (n, k))
    return a, b


def square_operands(size: int, seed: int = 1):
    """A, B bf16 ~ N(0,1)*0.1 from `seed` (config c4)."""
    g = torch.Generator().manual_seed(seed)
    a = _normal(g, (size, size), 0.1)
    b = _normal(g, (size, size), 0.1)
    return a, b


def normal_operands(m: int, n: int, k: int, seed: int, std_a: float, std_b: float):
    g = torch.Generator().manual_seed(seed)
    a = _normal(g, (m, k), std_a)
    b = _normal(g, (n, k), std_b)
    return a, b


def llm_operands(n: int, k: int, m: int = LLM_M, seed: int = 2):
    """Activations A ~ N(0,1) (M x K), weights B ~ N(0, 0.02) (N x K), seed 2 (config c5)."""
    return normal_operands(m, n, k, seed, 1.0, 0.02)


def llm_operands_device(n: int, k: int, device, m: int = LLM_M, seed: int = 2):
    """Config c5 drawn on the GPU: A ~ N(0,1) (M x K) then B ~ N(0, 0.02) (N x K),
    fp32 from a device ``torch.Generator`` seeded with `seed`, cast to bf16.

    Same distributions, shapes and draw order as ``llm_operands``; drawing on the
    device keeps the 128256 x 4096 weight matrix from costing every rank of a
    multi-GPU run ~20 s of host time. Every rank with the same seed and GPU
    model draws the same values.
    """
    g = torch.Generator(device=device).manual_seed(seed)
    a = (torch.randn((m, k), generator=g, device=device) * 1.0).to(torch.bfloat16)
    b = torch.empty((n, k), dtype=torch.bfloat16, device=device)
    step = max(1, (1 << 28) // max(k, 1))  # rows per fp32 draw (<= 1 GiB of fp32 at a time)
    for r in range(0, n, step):
        rows = min(step, n - r)
        b[r:r + rows] = (torch.randn((rows, k), generator=g, device=device) * 0.02).to(torch.bfloat16)
    return a, b


def ref_compat_available() -> bool:
    try:
        import cutlass  # noqa: F401
        import cutlass.torch  # noqa: F401
    except Exception:
        return False
    return True


def ref_compat_operands(m: int, n: int, k: int, seed: int = REF_SEED):
    """The reference's operands: torch.manual_seed(1111), then cutlass.torch.matrix for A, B.

    Returns host bf16 tensors A (M x K) and B (N x K), row-major.
    """
    import cutlass
    import cutlass.torch as cutlass_torch

    torch.manual_seed(seed)
    a = cutlass_torch.matrix(1, m, k, False, cutlass.BFloat16)
    b = cutlass_torch.matrix(1, n, k, False, cutlass.BFloat16)
    return a[:, :, 0].contiguous(), b[:, :, 0].contiguous()


def integer_operands(m: int, n: int, k: int, seed: int = REF_SEED):
    """Integer-valued operands in {-2..1} without the CUTLASS factory (exact fp32 sums)."""
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(-2, 2, (m, k), generator=g, dtype=torch.int32).to(torch.bfloat16)
    b = torch.randint(-2, 2, (n, k), generator=g, dtype=torch.int32).to(torch.bfloat16)
    return a, b
