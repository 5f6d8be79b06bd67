"""Multi-GPU layer: output-column (N) sharding of one GEMM over the ranks of a process group.

The reference has no multi-GPU path (its AGENTS.md rules out multi-GPU); this
layer is new. Each rank owns the output columns [n0, n1) given by
`b200_shard_range` (ceil(N/world) rounded up to 16 columns, the last shard
takes the remainder), holds A (M x K, replicated) and its B rows B[n0:n1], and
runs the single-GPU persistent kernel on them. The full matrix is produced
only when the caller asks for it:

  gather="none"    D shard M x (n1-n0) on this rank (weak-scaling path)
  gather="blocks"  NCCL all-gather of the padded shards into [world, M, W]
  gather="full"    the same, then one re-layout to row-major M x N
  p2p=True         fused gather: the GEMM's epilogue writes every output chunk
                   into every rank's row-major M x N buffer over NVLink (TMA
                   bulk stores, or 16-byte stores, through CUDA IPC mappings),
                   so the exchange overlaps the math tile by tile and needs no
                   re-layout; one NCCL all-reduce of a scalar then orders the ranks.
  engine="auto" (the default with p2p=True) picks "mc" on 8 or more GPUs when
                   a shard is at least 128 MiB, else "sm".
  p2p=True, engine="mc"
                   the multicast form of the fused gather: the full buffer is
                   torch symmetric memory bound to an NVLink multicast object,
                   and the epilogue writes each output chunk ONCE to the
                   multicast address; the NVSwitch replicates it into every
                   rank's buffer (each GPU sends its shard once, not once per peer).
  p2p=True, engine="ce"
                   the same buffers, but the GEMM writes only its own columns
                   and the copy engines then copy them into every peer's buffer
                   (one 2D copy per peer, each on its own stream), SMs idle.

One process per GPU; the process group is torch.distributed over NCCL (or
gloo for CPU tests of the host logic, with `local_gemm` injected).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from ._lib import shard_range

SHARD_GRANULE = 16


def shard_bounds(n: int, world: int, rank: int, granule: int = SHARD_GRANULE):
    return shard_range(n, world, rank, granule)


def shard_width(n: int, world: int, granule: int = SHARD_GRANULE) -> int:
    b, e = shard_bounds(n, world, 0, granule)
    return e - b


class _DeviceArray:
    """__cuda_array_interface__ view of a raw device allocation (int16 elements)."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<i2",
                                         "data": (int(ptr), False), "version": 3, "strides": None}


class PeerBuffer:
    """This rank's full-matrix output, mapped into every other rank (CUDA IPC)."""

    def __init__(self, m: int, n: int, group=None):
        self._lib = _lib.load()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        nbytes = m * n * 2
        hsize = int(self._lib.b200_ipc_handle_size())
        handle = ctypes.create_string_buffer(hsize)
        ptr = ctypes.c_void_p()
        _lib.check(self._lib.b200_peer_buffer_alloc(nbytes, ctypes.byref(ptr), handle),
                   "b200_peer_buffer_alloc", self._lib)
        self.ptr = int(ptr.value)
        self.tensor = torch.as_tensor(_DeviceArray(self.ptr, (m, n)),
                                      device=torch.device("cuda", torch.cuda.current_device())
                                      ).view(torch.bfloat16)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.raw), group=group)
        self.peers = {}
        for r, h in enumerate(handles):
            if r == self.rank:
                continue
            q = ctypes.c_void_p()
            _lib.check(self._lib.b200_peer_open(ctypes.create_string_buffer(h, hsize), ctypes.byref(q)),
                       "b200_peer_open", self._lib)
            self.peers[r] = int(q.value)

    def close(self):
        for q in self.peers.values():
            self._lib.b200_peer_close(ctypes.c_void_p(q))
        self.peers = {}
        if self.ptr:
            self._lib.b200_peer_buffer_free(ctypes.c_void_p(self.ptr))
            self.ptr = 0


class MulticastBuffer:
    """This rank's full-matrix output in torch symmetric memory, bound with every
    other rank's to one NVLink multicast object (multicast_ptr)."""

    def __init__(self, m: int, n: int, device, group=None):
        import torch.distributed._symmetric_memory as symm_mem
        grp = group if group is not None else dist.group.WORLD
        self.tensor = symm_mem.empty((m, n), dtype=torch.bfloat16, device=device)
        self._handle = symm_mem.rendezvous(self.tensor, grp)
        self.mc_ptr = int(self._handle.multicast_ptr)
        if self.mc_ptr == 0:
            raise RuntimeError("this GPU group has no NVLink multicast (NVLS) support")
        if self.mc_ptr % 16 != 0:
            raise RuntimeError("multicast mapping is not 16-byte aligned")
        self.peers = {}

    def close(self):
        self._handle = None
        self.tensor = None


class ShardedGemm:
    """D = A @ B^T with B (and D) split by output columns across the group."""

    def __init__(self, a: torch.Tensor, b_shard: torch.Tensor, n_total: int, *, group=None,
                 out_dtype=torch.bfloat16, mode: str = "auto", local_gemm=None, p2p: bool = False,
                 engine: str = "auto"):
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
        self.a, self.b = a, b_shard
        self._plan = None
        self.p2p = p2p
        if engine not in ("auto", "sm", "ce", "mc"):
            raise ValueError("engine must be 'auto', 'sm' (fused epilogue stores), 'mc' (fused "
                             "multicast stores) or 'ce' (copy engines)")
        requested = engine
        if engine == "auto":
            # Measured on B200 (8192 x N x 4096): multicast wins on 8 GPUs once each
            # rank's shard is large (263 MB: 3.71 vs 4.02 ms) and loses on small
            # shards and on 2 GPUs, where every GPU also receives its own shard back.
            shard_bytes = a.shape[0] * self.width * 2  # the common shard width: same on every rank
            engine = "mc" if (p2p and self.world >= 8 and shard_bytes >= (128 << 20)) else "sm"
        self.engine = engine
        self.peer_buffer = None
        if p2p:
            if local_gemm is not None or out_dtype != torch.bfloat16:
                raise ValueError("the fused gather runs the B200 kernel with bf16 output")
            if self.n_total % 8 != 0:
                raise ValueError("the fused gather needs N % 8 == 0 (16-byte rows)")
            if engine == "mc":
                try:
                    self.peer_buffer = MulticastBuffer(self.m, self.n_total, a.device, group)
                except RuntimeError:
                    if requested != "auto":
                        raise
                    engine = self.engine = "sm"  # no NVLS here: unicast peer stores
            if engine != "mc":
                self.peer_buffer = PeerBuffer(self.m, self.n_total, group)
            self.full = self.peer_buffer.tensor
            self.out = self.full[:, self.n0:self.n1]
        else:
            # Padded to the common shard width so the gather is one equal-size collective.
            self.block = torch.zeros((self.m, self.width), dtype=out_dtype, device=a.device)
            self.out = self.block[:, : self.n1 - self.n0]
        if local_gemm is None:
            from .gemm import GemmPlan
            if self.n1 > self.n0 and self.m > 0:
                self._plan = GemmPlan(a, b_shard, self.out, mode=mode)
                if p2p and engine == "mc":
                    self._plan.set_multicast(self.peer_buffer.mc_ptr + self.n0 * 2)
                if p2p and engine == "sm":
                    pitch_off = self.n0 * 2
                    self._plan.set_peers([self.peer_buffer.peers[r] + pitch_off
                                          for r in sorted(self.peer_buffer.peers)])
            self._local = self._plan.execute if self._plan is not None else (lambda: None)
        else:
            self._local = lambda: local_gemm(a, b_shard, self.out)
        self._flag = None

    @property
    def launches_per_step(self) -> int:
        return self._plan.launches_per_execute if self._plan is not None else 0

    def _copy_to_peers(self):
        """Copy-engine gather: this rank's columns into every peer's full buffer."""
        lib = self.peer_buffer._lib
        cur = torch.cuda.current_stream(self.a.device)
        if not hasattr(self, "_ce_streams"):
            self._ce_streams = [torch.cuda.Stream(self.a.device) for _ in self.peer_buffer.peers]
        done = torch.cuda.Event()
        done.record(cur)
        pitch = self.n_total * 2
        src = self.out.data_ptr()
        for s, r in zip(self._ce_streams, sorted(self.peer_buffer.peers)):
            s.wait_event(done)
            _lib.check(lib.b200_peer_copy_2d(self.peer_buffer.peers[r] + self.n0 * 2, pitch, src, pitch,
                                             (self.n1 - self.n0) * 2, self.m, s.cuda_stream),
                       "b200_peer_copy_2d", lib)
            ev = torch.cuda.Event()
            ev.record(s)
            cur.wait_event(ev)

    def run(self, gather: str = "none"):
        self._local()
        if self.p2p:
            if self.engine == "ce" and self.world > 1 and self.n1 > self.n0:
                self._copy_to_peers()
            # Order the ranks: after this all-reduce every rank's kernel (and its
            # peer writes, fenced system-wide before exit) has completed.
            if self._flag is None:
                self._flag = torch.zeros(1, dtype=torch.float32, device=self.a.device)
            if self.world > 1:
                dist.all_reduce(self._flag, group=self.group)
            return self.full if gather != "none" else self.out
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
        if self.peer_buffer is not None:
            # No rank may still be writing into a buffer that is about to go.
            torch.cuda.synchronize()
            if self.world > 1:
                dist.barrier(group=self.group)
            self.peer_buffer.close()
            self.peer_buffer = None
