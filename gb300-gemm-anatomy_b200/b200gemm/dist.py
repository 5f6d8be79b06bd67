"""Multi-GPU layer: output-column (N) sharding of one GEMM over the ranks of a process group.

The reference has no multi-GPU path (its AGENTS.md rules out multi-GPU); this
layer is new. Each rank owns the output columns [n0, n1) given by
`b200_shard_range` (ceil(N/world) rounded up to 16 columns, the last shard
takes the remainder), holds A (M x K, replicated) and its B rows B[n0:n1], and
runs the single-GPU persistent kernel on them. No collective runs unless the
caller asks for the full matrix:

  gather="none"    D shard M x (n1-n0) on this rank (weak-scaling path)
  gather="blocks"  NCCL all-gather of the padded shards into [world, M, W]
                   (W = shard width), one collective, no re-layout
  gather="full"    the same, then one re-layout to row-major M x N

One process per GPU; the process group is torch.distributed over NCCL (or
gloo for CPU tests of the host logic, with `local_gemm` injected).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ._lib import shard_range

SHARD_GRANULE = 16


def shard_bounds(n: int, world: int, rank: int, granule: int = SHARD_GRANULE):
    return shard_range(n, world, rank, granule)


def shard_width(n: int, world: int, granule: int = SHARD_GRANULE) -> int:
    b, e = shard_bounds(n, world, 0, granule)
    return e - b


class ShardedGemm:
    """D = A @ B^T with B (and D) split by output columns across the group."""

    def __init__(self, a: torch.Tensor, b_shard: torch.Tensor, n_total: int, *, group=None,
                 out_dtype=torch.bfloat16, mode: str = "auto", local_gemm=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.n_total = int(n_total)
        self.n0, self.n1 = shard_bounds(self.n_total, self.world, self.rank)
        if b_shard.shape[0] != self.n1 - self.n0:
            raise ValueError(f"rank {self.rank} owns columns [{self.n0}, {self.n1}) but B shard has "
                             f"{b_shard.shape[0]} rows")
        self.m = a.shape[0]
        self.width = shard_width(self.n_total, self.world)
        # Padded to the common shard width so the gather is one equal-size collective.
        self.block = torch.zeros((self.m, self.width), dtype=out_dtype, device=a.device)
        self.out = self.block[:, : self.n1 - self.n0]
        self.a, self.b = a, b_shard
        self._plan = None
        if local_gemm is None:
            from .gemm import GemmPlan
            if self.n1 > self.n0 and self.m > 0:
                self._plan = GemmPlan(a, b_shard, self.out, mode=mode)
            self._local = self._plan.execute if self._plan is not None else (lambda: None)
        else:
            self._local = lambda: local_gemm(a, b_shard, self.out)

    @property
    def launches_per_step(self) -> int:
        return self._plan.launches_per_execute if self._plan is not None else 0

    def run(self, gather: str = "none"):
        self._local()
        if gather == "none":
            return self.out
        if gather not in ("blocks", "full"):
            raise ValueError("gather must be 'none', 'blocks' or 'full'")
        blocks = torch.empty((self.world, self.m, self.width), dtype=self.block.dtype,
                             device=self.block.device)
        if self.world == 1:
            blocks[0].copy_(self.block)
        else:
            dist.all_gather_into_tensor(blocks.view(self.world * self.m, self.width), self.block,
                                        group=self.group)
        if gather == "blocks":
            return blocks
        full = blocks.permute(1, 0, 2).reshape(self.m, self.world * self.width)
        return full[:, : self.n_total].contiguous()

    def synchronize(self):
        if self._plan is not None:
            self._plan.synchronize()

    def destroy(self):
        if self._plan is not None:
            self._plan.destroy()
            self._plan = None
