"""CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use this
module, and only as the checker (or the timed CPU baseline); the product path
(libb200gemm.so, the b200gemm package) never imports it.

Two layers:
  * ctypes wrappers over oracle.c (built by oracle/Makefile into
    oracle/_build/liboracle.so): SplitMix64 pattern, word checksum, UMMA
    integer known answer, double/float GEMM.
  * numpy restatements of the same algorithms, cross-checked against the C
    code in the CPU tests, plus the reference's own CPU check arithmetic:
    reference_einsum (the fp32 IEEE einsum "mkl,nkl->mnl",
    src/gemm/gemm_comparison.py:2705-2722) run on the host.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"
PATTERN_SALT = 0xD1B54A32D192ED03
SPLITMIX_GAMMA = 0x9E3779B97F4A7C15
# Published first output of the SplitMix64 generator seeded with 0.
SPLITMIX_SEED0_FIRST = 0xE220A8397B1DCDAF
M64 = (1 << 64) - 1

_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.is_file():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.oracle_splitmix64.restype = ctypes.c_uint64
        L.oracle_splitmix64.argtypes = [ctypes.c_uint64]
        L.oracle_pattern_vectors.restype = None
        L.oracle_pattern_vectors.argtypes = [ctypes.c_uint64, ctypes.c_int64, ctypes.c_void_p]
        L.oracle_checksum_u32.restype = None
        L.oracle_checksum_u32.argtypes = [ctypes.c_void_p, ctypes.c_int64,
                                          ctypes.POINTER(ctypes.c_uint32),
                                          ctypes.POINTER(ctypes.c_uint64)]
        L.oracle_umma_reference.restype = None
        L.oracle_umma_reference.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        L.oracle_bf16_round.restype = ctypes.c_uint16
        L.oracle_bf16_round.argtypes = [ctypes.c_float]
        for name in ("oracle_gemm_tn_f64", "oracle_gemm_tn_f32"):
            fn = getattr(L, name)
            fn.restype = None
            fn.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                           ctypes.c_void_p, ctypes.c_void_p]
        _lib = L
    return _lib


# ----------------------------------------------------------------------------- C wrappers
def splitmix64(z: int) -> int:
    return int(lib().oracle_splitmix64(z & M64))


def pattern_words(start_vec: int, count: int) -> np.ndarray:
    """uint32[count*4]: the reference's 16-byte pattern vectors [start, start+count)."""
    out = np.empty(count * 4, dtype=np.uint32)
    lib().oracle_pattern_vectors(start_vec, count, out.ctypes.data)
    return out


def checksum_words(words: np.ndarray) -> tuple[int, int]:
    w = np.ascontiguousarray(words, dtype=np.uint32)
    x = ctypes.c_uint32(0)
    s = ctypes.c_uint64(0)
    lib().oracle_checksum_u32(w.ctypes.data, w.size, ctypes.byref(x), ctypes.byref(s))
    return int(x.value), int(s.value)


def umma_reference(cta_group: int, n: int, depth: int) -> np.ndarray:
    d = np.empty((128 * cta_group, n), dtype=np.float64)
    lib().oracle_umma_reference(cta_group, n, depth, d.ctypes.data)
    return d


def _bf16_bits(t) -> np.ndarray:
    """uint16 bit patterns of a bf16 torch tensor (or a uint16 array)."""
    if isinstance(t, np.ndarray):
        return np.ascontiguousarray(t, dtype=np.uint16)
    import torch
    return np.ascontiguousarray(t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16))


def gemm_tn_f64(a, b) -> np.ndarray:
    """D = A * B^T accumulated in double; a (M x K) and b (N x K) bf16."""
    ab, bb = _bf16_bits(a), _bf16_bits(b)
    m, k = ab.shape
    n = bb.shape[0]
    d = np.empty((m, n), dtype=np.float64)
    lib().oracle_gemm_tn_f64(m, n, k, ab.ctypes.data, bb.ctypes.data, d.ctypes.data)
    return d


def gemm_tn_f32(a, b) -> np.ndarray:
    ab, bb = _bf16_bits(a), _bf16_bits(b)
    m, k = ab.shape
    n = bb.shape[0]
    d = np.empty((m, n), dtype=np.float32)
    lib().oracle_gemm_tn_f32(m, n, k, ab.ctypes.data, bb.ctypes.data, d.ctypes.data)
    return d


# ----------------------------------------------------------------------------- numpy restatements
def np_splitmix64(z: np.ndarray) -> np.ndarray:
    z = z.astype(np.uint64)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def np_pattern_words(start_vec: int, count: int) -> np.ndarray:
    idx = np.arange(start_vec, start_vec + count, dtype=np.uint64)
    lo = np_splitmix64(idx)
    hi = np_splitmix64(idx ^ np.uint64(PATTERN_SALT))
    out = np.empty((count, 4), dtype=np.uint32)
    out[:, 0] = (lo & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    out[:, 1] = (lo >> np.uint64(32)).astype(np.uint32)
    out[:, 2] = (hi & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    out[:, 3] = (hi >> np.uint64(32)).astype(np.uint32)
    return out.reshape(-1)


def np_checksum_words(words: np.ndarray) -> tuple[int, int]:
    w = np.ascontiguousarray(words).view(np.uint32).reshape(-1)
    x = int(np.bitwise_xor.reduce(w)) if w.size else 0
    s = int(w.sum(dtype=np.uint64)) if w.size else 0
    return x, s & M64


def np_umma_reference(cta_group: int, n: int, depth: int) -> np.ndarray:
    r = np.arange(128 * cta_group)[:, None]
    kk = np.arange(16)[None, :]
    a = ((r + 3 * kk) % 7) - 3
    c = np.arange(n)[None, :]
    kc = np.arange(16)[:, None]
    b = ((2 * kc + c) % 5) - 2
    return depth * (a.astype(np.int64) @ b.astype(np.int64)).astype(np.float64)


def reference_einsum(a, b):
    """The reference's oracle math on the host: fp32 einsum 'mkl,nkl->mnl' with L = 1."""
    import torch
    a3 = a.to(torch.float32).unsqueeze(-1)
    b3 = b.to(torch.float32).unsqueeze(-1)
    return torch.einsum("mkl,nkl->mnl", a3, b3)[:, :, 0]
