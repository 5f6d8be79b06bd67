"""The oracle against the golden vectors (published constants and fixtures made
by running the reference's own Python code), and C vs numpy restatements."""
import json

import numpy as np
import pytest
import torch

from oracle import oracle


def test_splitmix_published_value(golden_dir):
    g = json.loads((golden_dir / "splitmix.json").read_text())
    assert oracle.splitmix64(oracle.SPLITMIX_GAMMA) == g["seed0_first_output"] == 0xE220A8397B1DCDAF
    assert int(oracle.np_splitmix64(np.array([oracle.SPLITMIX_GAMMA], dtype=np.uint64))[0]) == \
        0xE220A8397B1DCDAF
    assert oracle.pattern_words(0, 64).tolist() == g["pattern_words_0_64"]


@pytest.mark.parametrize("start,count", [(0, 1), (7, 1000), ((1 << 33) + 5, 257)])
def test_pattern_c_vs_numpy(start, count):
    assert np.array_equal(oracle.pattern_words(start, count), oracle.np_pattern_words(start, count))


def test_checksum_c_vs_numpy():
    w = np.random.default_rng(0).integers(0, 2 ** 32, size=100003, dtype=np.uint64).astype(np.uint32)
    assert oracle.checksum_words(w) == oracle.np_checksum_words(w)
    assert oracle.checksum_words(np.zeros(0, np.uint32)) == (0, 0)


@pytest.mark.parametrize("g", [1, 2])
@pytest.mark.parametrize("n", [64, 128, 256])
@pytest.mark.parametrize("depth", [4, 16, 32, 64, 128, 256])
def test_umma_known_answer(g, n, depth):
    d = oracle.umma_reference(g, n, depth)
    assert np.array_equal(d, oracle.np_umma_reference(g, n, depth))
    # spot values straight from the reference formulas (umma_1sm.cu:577-586)
    r, c = 5, 3
    s = sum((((r + 3 * k) % 7) - 3) * (((2 * k + c) % 5) - 2) for k in range(16))
    assert d[r, c] == depth * s


def test_gemm_oracle_matches_golden(golden_dir):
    z = np.load(golden_dir / "gemm_small.npz")
    for tag in ("128x256x64", "96x80x72", "200x264x136", "256x512x256"):
        a = torch.from_numpy(z[f"a_{tag}"]).view(torch.bfloat16)
        b = torch.from_numpy(z[f"b_{tag}"]).view(torch.bfloat16)
        ref = z[f"d_{tag}"].astype(np.float64)
        k = a.shape[1]
        d64 = oracle.gemm_tn_f64(a, b)
        assert np.abs(d64 - ref).max() <= k * 2.0 ** -22
        d32 = oracle.gemm_tn_f32(a, b)
        assert np.abs(d32 - ref).max() <= k * 2.0 ** -20
        assert torch.allclose(oracle.reference_einsum(a, b).double(), torch.from_numpy(ref))


def test_gemm_oracle_512_golden(golden_dir):
    from b200gemm import operands
    g = json.loads((golden_dir / "gemm_512.json").read_text())
    a, b = operands.uniform_operands(512, 512, 512, seed=0)
    d = oracle.gemm_tn_f64(a, b)
    idx = np.array(g["idx"])
    assert np.allclose(d[idx[:, 0], idx[:, 1]], g["values"], atol=512 * 2.0 ** -20)
    assert abs(d.sum() - g["sum"]) <= 1e-3 * abs(g["sumsq"]) ** 0.5 + 1e-3


def test_ref_compat_exact_in_oracle(golden_dir):
    z = np.load(golden_dir / "ref_small.npz")
    a = torch.from_numpy(z["a"]).view(torch.bfloat16)
    b = torch.from_numpy(z["b"]).view(torch.bfloat16)
    assert set(np.unique(a.float().numpy())) <= {-2.0, -1.0, 0.0, 1.0}
    assert np.array_equal(oracle.gemm_tn_f64(a, b), z["d"].astype(np.float64))


def test_bf16_round_rne():
    for f, expect in [(1.0, 0x3F80), (1.00390625, 0x3F80), (1.01171875, 0x3F82), (-2.5, 0xC020)]:
        assert oracle.lib().oracle_bf16_round(f) == expect
    x = torch.randn(1000, generator=torch.Generator().manual_seed(1))
    ours = np.array([oracle.lib().oracle_bf16_round(float(v)) for v in x], dtype=np.uint16)
    assert np.array_equal(ours, x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))
