"""Host-side plan policy without a GPU (b200_gemm_policy): mode AUTO, raster and
tile schedule for a 148-SM B200, pinned to the choices the GPU measurements
justified (each case names the measured reason)."""
import random

import pytest

from b200gemm import _lib, gemm


def pol(m, n, k, mode="auto", sm=148):
    return gemm.policy(m, n, k, mode=mode, sm_count=sm)


@pytest.fixture(autouse=True)
def _no_overrides(monkeypatch):
    for var in ("B200_GEMM_SCHEDULE", "B200_GEMM_RASTER", "B200_GEMM_GROUP"):
        monkeypatch.delenv(var, raising=False)


def test_bench_shape_runs_512x256_pair_tiles_dynamic():
    p = pol(8192, 8192, 8192)  # 512 tiles on 74 pairs = 6.92 waves, 25 % fewer L2->SM bytes
    assert (p["mode"], p["schedule"], p["tile_m"], p["num_tiles"], p["grid_ctas"]) == \
        ("2cta_m512", "dynamic", 512, 512, 148)
    assert p["raster_n"] == 0 and p["group"] == 8  # ~4096 A rows per raster group


def test_uneven_last_wave_takes_stream_k():
    p = pol(4096, 4096, 4096)  # 256 tiles = 3.46 waves
    assert (p["mode"], p["schedule"]) == ("2cta", "stream_k")
    assert (p["sk_groups"], p["sk_lanes"], p["sk_rounds"], p["sk_split_tiles"]) == (74, 1, 3, 34)


def test_skinny_grid_runs_stream_k_in_lanes():
    p = pol(32768, 512, 4096)  # 2 n-blocks: groups of two lanes share each A panel
    assert (p["schedule"], p["sk_lanes"], p["sk_lane_n"], p["sk_groups"]) == ("stream_k", 2, 1, 37)
    assert p["sk_split_tiles"] * 3 >= p["sk_groups"]


@pytest.mark.parametrize("shape", [(16384, 512, 4096), (512, 16384, 4096)])
def test_under_three_waves_stays_dynamic(shape):
    p = pol(*shape)  # 1.73 waves: stream-K measured 3 % slower
    assert (p["mode"], p["schedule"]) == ("2cta", "dynamic")


def test_small_problem_runs_one_cta_tiles():
    p = pol(512, 512, 512)
    assert (p["mode"], p["schedule"], p["grid_ctas"]) == ("1cta", "dynamic", 8)


@pytest.mark.parametrize("shape,raster_n,group", [
    ((8192, 4096, 4096), 1, 16),    # B 32 MiB fits L2: every n-block of an m-block in turn
    ((8192, 2048, 4096), 1, 8),
    ((16384, 512, 4096), 1, 2),
    ((8192, 14336, 4096), 0, 16),   # B 117 MiB: m-groups of ~4096 rows
    ((8192, 4096, 14336), 0, 9),    # K = 14336: groups capped to a 64 MiB A panel
    ((512, 16384, 4096), 0, 2),     # A is the narrow side: all m-blocks walk B
])
def test_raster_rule(shape, raster_n, group):
    p = pol(*shape)
    assert (p["raster_n"], p["group"]) == (raster_n, group)


def test_llm_shard_shape_takes_stream_k():
    p = pol(8192, 1792, 4096)  # 8-GPU shard of N = 14336: 3.03 waves (measured -6.6 %)
    assert p["schedule"] == "stream_k" and p["sk_rounds"] >= 2


def test_environment_overrides(monkeypatch):
    monkeypatch.setenv("B200_GEMM_SCHEDULE", "dynamic")
    assert pol(4096, 4096, 4096)["schedule"] == "dynamic"
    monkeypatch.setenv("B200_GEMM_SCHEDULE", "streamk")
    assert pol(16384, 512, 4096)["schedule"] == "stream_k"
    assert pol(8192, 8192, 8192)["schedule"] == "dynamic"  # 512x256 tiles never split
    monkeypatch.delenv("B200_GEMM_SCHEDULE")
    monkeypatch.setenv("B200_GEMM_RASTER", "m")
    monkeypatch.setenv("B200_GEMM_GROUP", "4")
    p = pol(8192, 4096, 4096)
    assert (p["raster_n"], p["group"]) == (0, 4)


def test_explicit_modes_and_invalid_arguments():
    assert pol(8192, 8192, 8192, mode="1cta")["tile_m"] == 128
    assert pol(8192, 8192, 8192, mode="2cta")["tile_m"] == 256
    lib = _lib.load()
    info = _lib.PolicyInfo()
    assert lib.b200_gemm_policy(0, 64, 64, 0, 148, info) == _lib.ERR_INVALID_ARGUMENT
    assert lib.b200_gemm_policy(64, 64, 64, 0, 1, info) == _lib.ERR_INVALID_ARGUMENT
    assert lib.b200_gemm_policy(64, 64, 60, 0, 148, info) == _lib.ERR_UNSUPPORTED  # K % 8
    assert lib.b200_gemm_policy(64, 64, 64, 9, 148, info) == _lib.ERR_INVALID_ARGUMENT
    assert lib.b200_gemm_policy(64, 64, 64, 0, 148, None) == _lib.ERR_INVALID_ARGUMENT


def test_invariants_over_random_shapes():
    """Every plan fits the GPU; stream-K only with one accumulator per tile, at least a
    third of a wave per split block, and (auto) three waves of work."""
    rng = random.Random(7)
    for _ in range(400):
        m = rng.randrange(8, 40000, 8)
        n = rng.randrange(8, 40000, 8)
        k = rng.randrange(8, 20000, 8)
        sm = rng.choice([148, 132, 120, 16])
        p = pol(m, n, k, sm=sm)
        cta = 1 if p["mode"] == "1cta" else 2
        assert 0 < p["grid_ctas"] <= sm and p["grid_ctas"] % cta == 0
        assert p["num_tiles"] == p["num_m_blocks"] * p["num_n_blocks"]
        if p["schedule"] == "stream_k":
            assert p["mode"] in ("1cta", "2cta")
            assert p["waves"] >= 3.0
            assert p["sk_split_tiles"] * 3 >= p["sk_groups"]
            assert p["sk_rounds"] >= 1
            assert p["sk_groups"] * p["sk_lanes"] * cta == p["grid_ctas"]
