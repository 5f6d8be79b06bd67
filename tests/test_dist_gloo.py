"""Host logic of the N-sharded multi-GPU layer on CPU ranks (gloo, world size 2 and 3).

The local GEMM is injected (the CPU oracle) so the shard bounds, padding,
all-gather and re-layout run exactly as on GPUs without one.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, n, m, k, q):
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(repo / "gb300-gemm-anatomy_b200"))
    sys.path.insert(0, str(repo))
    from b200gemm import dist as bdist, operands
    from oracle import oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _body(rank, world, n, m, k, q)
    except Exception as exc:  # report instead of leaving the parent waiting
        q.put((rank, False, repr(exc)))
    finally:
        dist.destroy_process_group()


def _body(rank, world, n, m, k, q):
    from b200gemm import dist as bdist, operands
    from oracle import oracle
    if True:
        a, b = operands.uniform_operands(m, n, k, seed=9)
        n0, n1 = bdist.shard_bounds(n, world, rank)

        def local(a_, b_, out):
            if b_.shape[0]:
                out.copy_(torch.from_numpy(oracle.gemm_tn_f64(a_, b_)).to(out.dtype))

        sg = bdist.ShardedGemm(a, b[n0:n1].contiguous(), n, out_dtype=torch.float32,
                               local_gemm=local)
        shard = sg.run("none").clone()
        full = sg.run("full")
        blocks = sg.run("blocks")
        ref = torch.from_numpy(oracle.gemm_tn_f64(a, b)).float()
        ok = bool(torch.equal(full, ref)) and bool(torch.equal(shard, ref[:, n0:n1]))
        ok = ok and tuple(blocks.shape) == (world, m, bdist.shard_width(n, world))
        q.put((rank, ok, (n0, n1)))


@pytest.mark.parametrize("world,n", [(2, 96), (2, 100), (3, 64), (2, 8)])
def test_sharded_gather_matches_full_gemm(world, n):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, 24, 32, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=60) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    assert all(ok for _, ok, _ in results), results
    bounds = [r[2] for r in results]
    assert bounds[0][0] == 0 and bounds[-1][1] == n
    assert all(bounds[i][1] == bounds[i + 1][0] for i in range(world - 1))


def test_llm_shard_widths():
    from b200gemm import dist as bdist
    assert bdist.shard_width(128256, 8) == 16032
    assert [bdist.shard_bounds(128256, 8, r) for r in (0, 7)] == [(0, 16032), (112224, 128256)]
    assert bdist.shard_width(14336, 8) == 1792
