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
    p = pol(4096, 4096, 4096, mode="2cta_n128")  # 512 tiles of 256 x 128, never split along K
    assert (p["tile_m"], p["tile_n"], p["num_tiles"], p["schedule"]) == (256, 128, 512, "dynamic")
    lib = _lib.load()
    info = _lib.PolicyInfo()
    assert lib.b200_gemm_policy(0, 64, 64, 0, 148, info) == _lib.ERR_INVALID_ARGUMENT
    assert lib.b200_gemm_policy(64, 64, 64, 0, 1, info) == _lib.ERR_INVALID_ARGUMENT
    assert lib.b200_gemm_policy(64, 64, 60, 0, 148, info) == _lib.ERR_UNSUPPORTED  # K % 8
    assert lib.b200_gemm_policy(64, 64, 64, 9, 148, info) == _lib.ERR_INVALID_ARGUMENT
    assert lib.b200_gemm_policy(64, 64, 64, 5, 148, info) == _lib.ERR_INVALID_ARGUMENT
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


def _sk_walk(p):
    """Restatement of the kernel's stream-K walk (sk_begin / sk_next in
    csrc/gemm_sm100.cu): per group, the split-block items from its last
    super-tile down to its first, then its whole-tile rounds."""
    nk, groups = p["num_k_blocks"], p["sk_groups"]
    iters = p["sk_split_tiles"] * nk
    start = [g * iters // groups for g in range(groups + 1)]
    walks = []
    for g in range(groups):
        lo, hi, items = start[g], start[g + 1], []
        while lo < hi:
            tl = (hi - 1) // nk
            a = max(lo, tl * nk)
            kb0, kb1 = a - tl * nk, hi - tl * nk
            role = 1 if kb1 < nk else (2 if kb0 > 0 else 0)
            items.append((tl, kb0, kb1, role))
            hi = a
        for r in range(p["sk_rounds"]):
            items.append((p["sk_split_tiles"] + r * groups + g, 0, nk, 0))
        walks.append(items)
    return walks, start


@pytest.mark.parametrize("shape,mode,sm", [
    ((4096, 4096, 4096), "auto", 148), ((32768, 512, 4096), "auto", 148),
    ((8192, 1792, 4096), "auto", 148), ((2304, 2304, 1024), "2cta", 148),
    ((4096, 4096, 4096), "1cta", 148), ((5376, 2816, 4096), "auto", 132),
    ((2560, 2560, 1000), "1cta", 16),
])
def test_stream_k_walk_covers_every_slice_and_waits_only_downward(monkeypatch, shape, mode, sm):
    """Every k-slice of every super-tile is computed exactly once; a finisher only
    waits for groups with a lower index (dispatched before it), so the schedule
    completes even when not every cluster of the grid is resident."""
    monkeypatch.setenv("B200_GEMM_SCHEDULE", "streamk")
    p = pol(*shape, mode=mode, sm=sm)
    assert p["schedule"] == "stream_k"
    nk = p["num_k_blocks"]
    walks, start = _sk_walk(p)
    supers = p["sk_split_tiles"] + p["sk_rounds"] * p["sk_groups"]
    seen = {}
    for g, items in enumerate(walks):
        split = [it for it in items if it[0] < p["sk_split_tiles"]]
        writers = [i for i, it in enumerate(split) if it[3] == 1]
        finishers = [i for i, it in enumerate(split) if it[3] == 2]
        assert len(writers) <= 1 and len(finishers) <= 1
        if writers:
            assert writers[0] == 0  # the partial is produced first
        if finishers:
            assert finishers[0] == len(split) - 1  # the cut tile is finished last
        for (t, kb0, kb1, role) in items:
            for kb in range(kb0, kb1):
                assert (t, kb) not in seen
                seen[(t, kb)] = g
            if role == 2:
                tile_start = t * nk
                deps = [w for w in range(g) if start[w + 1] > tile_start and start[w] < tile_start + nk]
                assert deps and max(deps) < g
                assert all(walks[w][0][0] == t and walks[w][0][3] == 1 for w in deps)
    assert len(seen) == supers * nk
    assert max(t for t, _ in seen) == supers - 1
