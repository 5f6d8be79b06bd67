"""Memory-path layer front end: LDGSTS / TMA global->SMEM streaming plans.

Replaces the reference's `ldgsts` and `tma` binaries (src/memory/ldgsts.cu,
src/memory/tma.cu) as a library: a plan over a device buffer, launched in one
of three modes (validate against the SplitMix64 pattern, full checksum, or the
reference's timed sink mode). Geometry follows the reference:
  stage_bytes = bytes_in_flight_per_sm / stages  (ldgsts.cu:18-20, 193-201)
and adds CTAs/SM in {1, 2, 4}.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

METHODS = {"ldgsts": _lib.STREAM_LDGSTS, "tma": _lib.STREAM_TMA, "tma_sw128": _lib.STREAM_TMA_SW128}
MODES = {"validate": _lib.STREAM_VALIDATE, "checksum": _lib.STREAM_CHECKSUM, "sink": _lib.STREAM_SINK}
REF_STAGES = (2, 4, 8)
REF_BIF_KIB = (16, 32, 64)
CTAS_PER_SM = (1, 2, 4)


def stage_bytes_for(bytes_in_flight_kib: int, stages: int) -> int:
    """The reference's stage size: bytes in flight per SM split evenly over the ring."""
    return bytes_in_flight_kib * 1024 // stages


def fill_pattern(buf: torch.Tensor, stream=None) -> None:
    """Write the reference's SplitMix64 index pattern over the whole buffer."""
    lib = _lib.load()
    nbytes = buf.numel() * buf.element_size()
    s = torch.cuda.current_stream(buf.device) if stream is None else stream
    _lib.check(lib.b200_fill_pattern(buf.data_ptr(), nbytes, int(s.cuda_stream)),
               "b200_fill_pattern", lib)


class StreamPlan:
    def __init__(self, buf: torch.Tensor, method: str, stages: int, stage_bytes: int,
                 ctas_per_sm: int = 1, passes: int = 1, rotation: int = 0):
        self._lib = _lib.load()
        if buf.device.type != "cuda" or not buf.is_contiguous():
            raise ValueError("buf must be a contiguous CUDA tensor")
        if method not in METHODS:
            raise ValueError(f"method must be one of {sorted(METHODS)}")
        self.buf = buf
        self.nbytes = buf.numel() * buf.element_size()
        self.cfg = _lib.StreamConfig(METHODS[method], stages, stage_bytes, ctas_per_sm, passes,
                                     rotation)
        plan = ctypes.c_void_p(None)
        info = _lib.StreamResult()
        rc = self._lib.b200_stream_plan_create(ctypes.byref(self.cfg), buf.data_ptr(), self.nbytes,
                                               buf.device.index or 0, ctypes.byref(plan),
                                               ctypes.byref(info))
        _lib.check(rc, "b200_stream_plan_create", self._lib)
        self._plan = plan
        self.info = {n: getattr(info, n) for n, _ in _lib.StreamResult._fields_}

    def execute(self, mode: str = "sink", stream=None) -> None:
        s = torch.cuda.current_stream(self.buf.device) if stream is None else stream
        _lib.check(self._lib.b200_stream_plan_execute(self._plan, MODES[mode], int(s.cuda_stream)),
                   "b200_stream_plan_execute", self._lib)

    def result(self, stream=None) -> dict:
        s = torch.cuda.current_stream(self.buf.device) if stream is None else stream
        out = _lib.StreamResult()
        _lib.check(self._lib.b200_stream_plan_result(self._plan, int(s.cuda_stream),
                                                     ctypes.byref(out)),
                   "b200_stream_plan_result", self._lib)
        r = {n: getattr(out, n) for n, _ in _lib.StreamResult._fields_}
        r["checksum_xor"] &= 0xFFFFFFFF
        r["checksum_sum"] &= (1 << 64) - 1
        return r

    def destroy(self) -> None:
        if getattr(self, "_plan", None) is None:
            return
        plan, self._plan = self._plan, None
        _lib.check(self._lib.b200_stream_plan_destroy(plan), "b200_stream_plan_destroy", self._lib)

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


def device_checksum(buf: torch.Tensor, method: str = "ldgsts", stages: int = 4,
                    stage_bytes: int = 16384, ctas_per_sm: int = 1) -> tuple[int, int]:
    """(xor32, sum64) of every 32-bit word of `buf`, computed by a streaming kernel."""
    plan = StreamPlan(buf, method, stages, stage_bytes, ctas_per_sm)
    try:
        plan.execute("checksum")
        r = plan.result()
    finally:
        plan.destroy()
    return r["checksum_xor"], r["checksum_sum"]
