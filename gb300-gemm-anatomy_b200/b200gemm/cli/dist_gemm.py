"""N-sharded GEMM across the GPUs of one node, with the three gather choices timed.

Run one process per GPU (torchrun --nproc-per-node G ... -m b200gemm.cli.dist_gemm).
Config: M=8192 activations ~ N(0,1), weights ~ N(0,0.02), seed 2 (the LLM
projection config), drawn on the device; every rank draws the same global B
from the seed and keeps its shard. For each shape it checks the gathered D against a torch fp32
reference on sampled rows, then times (CUDA events, max over ranks):
  none   the sharded GEMM alone (weak scaling of the compute)
  nccl   GEMM, then NCCL all-gather of the bf16 shards and the re-layout
  p2p    the fused gather: the GEMM epilogue TMA-stores every tile to every peer
  p2p_st the fused gather with per-thread 16-byte stores instead of TMA
  ce     GEMM, then the copy engines copy this rank's columns into every peer's
         full buffer (no SM work, no re-layout)
  mc     the fused gather through NVLink multicast: each output chunk is written
         once to a multicast address and the switch replicates it to every GPU
Prints one CSV row per (shape, gather) on rank 0.
"""
from __future__ import annotations

import argparse
import os
import sys

SHAPES = ((4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="dist_gemm")
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--shape", action="append", help="NxK (repeatable); default: the LLM shapes")
    ap.add_argument("--iterations", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--gathers", default="none,nccl,p2p,mc,ce")
    args = ap.parse_args(argv)
    import torch
    import torch.distributed as dist

    from .. import dist as bdist, operands

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl" if world > 1 else "gloo", device_id=dev if world > 1 else None)
    shapes = [tuple(int(x) for x in s.split("x")) for s in args.shape] if args.shape else SHAPES
    rows = []
    for (n, k) in shapes:
        torch.backends.cuda.matmul.allow_tf32 = False
        a, b_full = operands.llm_operands_device(n, k, dev, m=args.m)
        n0, n1 = bdist.shard_bounds(n, world, rank)
        b = b_full[n0:n1].contiguous()
        idx = torch.arange(0, args.m, max(args.m // 64, 1), device=dev)
        ref = (a[idx].float() @ b_full.float().T).cpu()
        del b_full
        for gather in args.gathers.split(","):
            # p2p: fused gather with TMA bulk stores to the peers; p2p_st: 16-byte stores.
            if gather == "p2p_st":
                os.environ["B200_PEER_STORES"] = "st"
            else:
                os.environ.pop("B200_PEER_STORES", None)
            sg = bdist.ShardedGemm(a, b, n, p2p=gather.startswith("p2p") or gather in ("ce", "mc"),
                                   engine=gather if gather in ("ce", "mc") else "sm")
            mode = "none" if gather == "none" else "full"
            full = sg.run(mode)
            torch.cuda.synchronize()
            if gather != "none":
                got = full[idx].float().cpu()
                rel = float((got - ref).norm() / ref.norm())
                if rel > 1e-2:
                    raise RuntimeError(f"{n}x{k} {gather}: rel err {rel}")
            for _ in range(args.warmup):
                sg.run(mode)
            torch.cuda.synchronize()
            dist.barrier()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.iterations):
                sg.run(mode)
            e1.record()
            torch.cuda.synchronize()
            ms = torch.tensor([e0.elapsed_time(e1) / args.iterations], device=dev)
            if world > 1:
                dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            sg.synchronize()
            sg.destroy()
            t = float(ms.item())
            flop = 2.0 * args.m * n * k
            gather_bytes = args.m * (n1 - n0) * 2 * (world - 1)
            rows.append((n, k, gather, world, t, flop / t / 1e9, gather_bytes / t / 1e6))
            del full
            torch.cuda.empty_cache()
    if rank == 0:
        print("m,n,k,gather,n_gpus,ms,tflops_total,sent_gbps_per_gpu")
        for (n, k, gather, w, t, tf, gbps) in rows:
            print(f"{args.m},{n},{k},{gather},{w},{t:.4f},{tf:.1f},{gbps:.1f}")
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
