"""Memory-path streamers on the GPU: bit-exact against the oracle.

VALIDATE mode compares every 16-byte vector with the SplitMix64 pattern
(0 mismatches required); CHECKSUM mode must equal the oracle's XOR/sum of the
same bytes exactly; SINK mode must equal the host recomputation of the
reference's per-thread sink word.
"""
import numpy as np
import pytest
import torch

from b200gemm import memory_paths as mp
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def sm_count():
    return torch.cuda.get_device_properties(0).multi_processor_count


@pytest.fixture(scope="module")
def pattern_buf():
    # 8 x (148 x 32 KiB) like the reference self-test (ldgsts.cu:75,474-478), plus a ragged tail.
    nbytes = 8 * sm_count() * 32 * 1024 + 64 * 1024
    buf = torch.empty(nbytes // 2, dtype=torch.int16, device=DEV)
    mp.fill_pattern(buf)
    torch.cuda.synchronize()
    return buf


def test_fill_pattern_matches_oracle(pattern_buf):
    words = pattern_buf[: 4096 * 8].view(torch.int32).cpu().numpy().view(np.uint32)
    assert np.array_equal(words, oracle.pattern_words(0, words.size // 4))


@pytest.mark.parametrize("method", ["ldgsts", "tma", "tma_sw128"])
@pytest.mark.parametrize("stages", [2, 4, 8])
@pytest.mark.parametrize("bif_kib", [16, 32, 64])
def test_reference_grid_validate(pattern_buf, method, stages, bif_kib):
    sb = mp.stage_bytes_for(bif_kib, stages)
    nbytes = (pattern_buf.numel() * 2 // sb) * sb
    buf = pattern_buf[: nbytes // 2]
    if method == "tma_sw128" and sb % 4096:
        # each warp's quarter of a swizzled stage must hold whole 1024-byte atoms
        with pytest.raises(mp._lib.BridgeError):
            mp.StreamPlan(buf, method, stages, sb)
        return
    plan = mp.StreamPlan(buf, method, stages, sb, ctas_per_sm=1, passes=2, rotation=3)
    plan.execute("validate")
    r = plan.result()
    plan.destroy()
    assert r["status"] == 0 and r["mismatches"] == 0
    assert r["occupancy_ctas_per_sm"] == 1


@pytest.mark.parametrize("method", ["ldgsts", "tma", "tma_sw128"])
@pytest.mark.parametrize("ctas", [1, 2, 4])
@pytest.mark.parametrize("stages", [2, 4, 8])
def test_ctas_per_sm_checksum(pattern_buf, method, ctas, stages):
    sb = 8192 if stages * 8192 * ctas <= 200 * 1024 else 4096
    nbytes = (pattern_buf.numel() * 2 // sb) * sb
    buf = pattern_buf[: nbytes // 2]
    plan = mp.StreamPlan(buf, method, stages, sb, ctas_per_sm=ctas, passes=1)
    assert plan.info["occupancy_ctas_per_sm"] == ctas
    plan.execute("checksum")
    r = plan.result()
    plan.destroy()
    host = buf.view(torch.int32).cpu().numpy().view(np.uint32)
    assert (r["checksum_xor"], r["checksum_sum"]) == oracle.checksum_words(host)


def test_seeded_bf16_checksum():
    g = torch.Generator().manual_seed(11)
    host = (torch.rand(3 * 1024 * 1024 + 4096, generator=g) * 2 - 1).to(torch.bfloat16)
    buf = host.to(DEV)
    x, s = mp.device_checksum(buf, "tma_sw128", stages=4, stage_bytes=8192)
    assert (x, s) == oracle.checksum_words(host.view(torch.int16).numpy().view(np.uint32))


def test_sink_matches_host(pattern_buf):
    """SINK: XOR over all threads of the first word each thread touches per tile."""
    sb = 4096
    nbytes = sm_count() * 4 * sb
    buf = pattern_buf[: nbytes // 2]
    plan = mp.StreamPlan(buf, "ldgsts", 4, sb, ctas_per_sm=1, passes=1)
    plan.execute("sink")
    r = plan.result()
    plan.destroy()
    w = buf.view(torch.int32).cpu().numpy().view(np.uint32).reshape(-1, sb // 4)
    # thread t reads word 4*t of every tile; XOR over everything
    expect = int(np.bitwise_xor.reduce(w[:, 0:128 * 4:4].reshape(-1)))
    assert r["sink_xor"] == expect


def test_invalid_configs(pattern_buf):
    with pytest.raises(mp._lib.BridgeError):
        mp.StreamPlan(pattern_buf, "ldgsts", 3, 8192)
    with pytest.raises(mp._lib.BridgeError):
        mp.StreamPlan(pattern_buf, "ldgsts", 8, 65536, ctas_per_sm=4)


@pytest.mark.parametrize("method", ["tma", "tma_sw128"])
def test_tma_sink_matches_host(pattern_buf, method):
    """TMA SINK: warp w, lane l reads word 0 of vector l of quarter w of each stage."""
    sb = 8192
    nbytes = sm_count() * 4 * sb
    buf = pattern_buf[: nbytes // 2]
    plan = mp.StreamPlan(buf, method, 4, sb, ctas_per_sm=1, passes=1)
    plan.execute("sink")
    r = plan.result()
    plan.destroy()
    w = buf.view(torch.int32).cpu().numpy().view(np.uint32).reshape(-1, 4, sb // 64, 4)
    # quarter q, 16-byte slot l (l < 32) in shared memory; with the 128-byte swizzle
    # slot l holds vector (l >> 3) * 8 + ((l & 7) ^ ((l >> 3) & 7)) of the quarter
    lanes = np.arange(32)
    vec = lanes if method == "tma" else (lanes >> 3) * 8 + ((lanes & 7) ^ ((lanes >> 3) & 7))
    expect = int(np.bitwise_xor.reduce(w[:, :, vec, 0].reshape(-1)))
    assert r["sink_xor"] == expect
