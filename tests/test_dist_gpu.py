"""N-sharded GEMM on every visible GPU (skipped with fewer than 2).

Each rank runs the B200 kernel on its output columns; the full matrix is
gathered with one NCCL all-gather, by the kernel itself (fused gather: peer
stores over NVLink, or multicast stores through an NVLS object where the node
has one), or by the copy engines, and compared on every rank with the CPU
oracle. NCCL's own NVLS is off (NCCL_NVLS_ENABLE=0); every rank stays up for
the whole test (no rank leaves while its memory is bound to a multicast object).
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(repo / "gb300-gemm-anatomy_b200"))
    sys.path.insert(0, str(repo))
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from b200gemm import check, dist as bdist, operands
        from oracle import oracle
        m, n, k = 384, 1000, 256
        a, b = operands.uniform_operands(m, n, k, seed=12)
        n0, n1 = bdist.shard_bounds(n, world, rank)
        ref = torch.from_numpy(oracle.gemm_tn_f64(a, b))
        for p2p, stores in ((False, None), (True, "tma"), (True, "st")):
            if stores == "st":
                os.environ["B200_PEER_STORES"] = "st"
            else:
                os.environ.pop("B200_PEER_STORES", None)
            for mode in ("2cta", "2cta_m512", "1cta"):
                sg = bdist.ShardedGemm(a.to(dev), b[n0:n1].contiguous().to(dev), n, mode=mode,
                                       p2p=p2p)
                for _ in range(2):  # twice: the second launch reuses the plan and buffers
                    full = sg.run("full")
                    sg.synchronize()
                    torch.cuda.synchronize()
                    check.bf16_tolerance_check(f"rank {rank} p2p={p2p} {mode}", ref, full.cpu(), k,
                                               1.0, 1.0)
                sg.destroy()
        # The multicast form of the fused gather (NVLS), where the node has it;
        # copy-engine gather always.
        os.environ.pop("B200_PEER_STORES", None)
        for engine in ("mc", "ce"):
            for mode in ("2cta", "2cta_m512", "1cta"):
                try:
                    sg = bdist.ShardedGemm(a.to(dev), b[n0:n1].contiguous().to(dev), n, mode=mode,
                                           p2p=True, engine=engine)
                except RuntimeError as exc:
                    if engine == "mc" and "multicast" in str(exc):
                        break  # no NVLS on this node: nothing to check for this engine
                    raise
                for _ in range(2):
                    full = sg.run("full")
                    sg.synchronize()
                    torch.cuda.synchronize()
                    check.bf16_tolerance_check(f"rank {rank} engine={engine} {mode}", ref, full.cpu(),
                                               k, 1.0, 1.0)
                sg.destroy()
        # Stream-K per shard (forced): cut tiles are finished by the epilogue that
        # also sends the output chunks to the peers.
        os.environ.pop("B200_PEER_STORES", None)
        os.environ["B200_GEMM_SCHEDULE"] = "streamk"
        try:
            m2, n2, k2 = 2304, 2304 * world, 1024
            a2, b2 = operands.uniform_operands(m2, n2, k2, seed=13)
            s0, s1 = bdist.shard_bounds(n2, world, rank)
            a2d, b2d = a2.to(dev), b2.to(dev)
            ref2 = (a2d.double() @ b2d.double().T).cpu()
            for p2p in (False, True):
                sg = bdist.ShardedGemm(a2d, b2d[s0:s1].contiguous(), n2, mode="2cta", p2p=p2p)
                assert sg._plan.schedule == "stream_k", sg._plan.schedule
                for _ in range(2):
                    full = sg.run("full")
                    sg.synchronize()
                    torch.cuda.synchronize()
                    check.bf16_tolerance_check(f"rank {rank} p2p={p2p} stream-K", ref2, full.cpu(),
                                               k2, 1.0, 1.0)
                sg.destroy()
        finally:
            os.environ.pop("B200_GEMM_SCHEDULE", None)
        q.put((rank, True, ""))
    except Exception as exc:
        q.put((rank, False, repr(exc)))
    finally:
        dist.destroy_process_group()


def test_sharded_gemm_nccl_gather():
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs at least 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res), res
