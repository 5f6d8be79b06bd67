"""GEMM candidate front end: plans over the C ABI, torch tensors in and out.

``B200GemmBridge`` has the same life cycle and error behaviour as the
reference driver's ``CublasLtBridge`` (``src/gemm/gemm_comparison.py:1299-1460``):
one plan at a time, ``create_plan`` -> ``execute`` -> ``synchronize`` ->
``destroy``, a non-zero return code raises ``BridgeError`` with the library's
diagnostic. ``gemm()`` is the one-call convenience used by the drivers, the
bench and the multi-GPU layer.

Layout contract (TN, ``gemm_comparison.py:2670-2691``): ``a`` is M x K
row-major, ``b`` is N x K row-major, the result is ``a @ b.T`` (M x N).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import BridgeError

_DTYPE_CODE = {torch.bfloat16: _lib.OUT_BF16, torch.float32: _lib.OUT_F32}
_MODE_CODE = {"auto": _lib.MODE_AUTO, "1cta": _lib.MODE_1CTA, "2cta": _lib.MODE_2CTA,
              "2cta_m512": _lib.MODE_2CTA_M512, "2cta_n128": _lib.MODE_2CTA_N128}


def _stream_handle(stream) -> int:
    if stream is None:
        stream = torch.cuda.current_stream()
    return int(stream.cuda_stream) if hasattr(stream, "cuda_stream") else int(stream)


def _require_operand(t: torch.Tensor, name: str, shape) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must live on a CUDA device, got {t.device}")
    if t.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be bfloat16, got {t.dtype}")
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")
    if t.numel() and (t.stride(-1) != 1 or (t.dim() == 2 and t.stride(0) != t.shape[1])):
        raise ValueError(f"{name} must be row-major contiguous (K innermost), strides {t.stride()}")


class GemmPlan:
    """One planned GEMM over fixed device buffers (the plan holds raw pointers)."""

    def __init__(self, a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, *, mode: str = "auto",
                 stream=None, ldd: int | None = None):
        self._lib = _lib.load()
        m, k = a.shape
        n = b.shape[0]
        _require_operand(a, "A", (m, k))
        _require_operand(b, "B", (n, k))
        if out.dtype not in _DTYPE_CODE:
            raise ValueError(f"output dtype must be bfloat16 or float32, got {out.dtype}")
        if out.device != a.device or b.device != a.device:
            raise ValueError("A, B and D must be on the same device")
        ldd = int(out.stride(0)) if ldd is None else int(ldd)
        if out.dim() != 2 or out.shape[0] != m or out.shape[1] != n or out.stride(1) != 1:
            raise ValueError(f"D must be an M x N row-major view, got shape {tuple(out.shape)} "
                             f"strides {out.stride()}")
        if mode not in _MODE_CODE:
            raise ValueError(f"mode must be one of {sorted(_MODE_CODE)}")
        self.a, self.b, self.out = a, b, out  # keep the buffers alive
        self.m, self.n, self.k = int(m), int(n), int(k)
        self.stream = _stream_handle(stream)
        plan = ctypes.c_void_p(None)
        info = _lib.PlanInfo()
        with torch.cuda.device(a.device):
            rc = self._lib.b200_gemm_plan_create_ex(
                self.m, self.n, self.k, a.data_ptr(), b.data_ptr(), out.data_ptr(), ldd,
                _DTYPE_CODE[out.dtype], _MODE_CODE[mode], self.stream, ctypes.byref(plan),
                ctypes.byref(info))
        _lib.check(rc, "b200_gemm_plan_create_ex", self._lib)
        self._plan = plan
        self.info = {name: getattr(info, name) for name, _ in _lib.PlanInfo._fields_}

    @property
    def launches_per_execute(self) -> int:
        return int(self._lib.b200_gemm_plan_launches(self._plan))

    @property
    def schedule(self) -> str:
        """'dynamic' (whole tiles from a global counter) or 'stream_k'."""
        return "stream_k" if self._lib.b200_gemm_plan_schedule(self._plan) == 1 else "dynamic"

    def set_peers(self, peer_ptrs) -> None:
        """Fused gather: also write every output chunk into these peer buffers."""
        arr = (ctypes.c_void_p * max(len(peer_ptrs), 1))(*[ctypes.c_void_p(int(q)) for q in peer_ptrs])
        _lib.check(self._lib.b200_gemm_plan_set_peers(self._plan, len(peer_ptrs), arr),
                   "b200_gemm_plan_set_peers", self._lib)

    def set_multicast(self, mc_ptr: int) -> None:
        """Multicast gather: also write every output chunk once to this NVLink
        multicast address (this shard's first column of the full D); 0 = off."""
        _lib.check(self._lib.b200_gemm_plan_set_multicast(self._plan, ctypes.c_void_p(int(mc_ptr) or None)),
                   "b200_gemm_plan_set_multicast", self._lib)

    TRACE_SLOTS = 64

    def enable_trace(self) -> torch.Tensor:
        """Allocate and attach a per-CTA timeline buffer (see b200_gemm_plan_set_trace)."""
        buf = torch.zeros((max(self.info["grid_ctas"], 1), self.TRACE_SLOTS), dtype=torch.int64,
                          device=self.a.device)
        _lib.check(self._lib.b200_gemm_plan_set_trace(self._plan, buf.data_ptr(), self.TRACE_SLOTS),
                   "b200_gemm_plan_set_trace", self._lib)
        self._trace = buf
        return buf

    def execute(self, stream=None) -> None:
        if self._plan is None:
            raise BridgeError("the plan was destroyed")
        if stream is None:
            rc = self._lib.b200_gemm_plan_execute(self._plan)
        else:
            rc = self._lib.b200_gemm_plan_execute_on(self._plan, _stream_handle(stream))
        _lib.check(rc, "b200_gemm_plan_execute", self._lib)

    def synchronize(self) -> None:
        if self._plan is None:
            raise BridgeError("the plan was destroyed")
        _lib.check(self._lib.b200_stream_synchronize(self._plan), "b200_stream_synchronize",
                   self._lib)

    def destroy(self) -> None:
        if getattr(self, "_plan", None) is None:
            return
        plan, self._plan = self._plan, None
        _lib.check(self._lib.b200_gemm_plan_destroy(plan), "b200_gemm_plan_destroy", self._lib)

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class B200GemmBridge:
    """Drop-in for the reference's ``CublasLtBridge`` plan life cycle.

    ``create_plan(m, n, k, a_ptr, b_ptr, c_ptr, d_ptr, stream)`` takes the same
    arguments as ``CublasLtBridge.create_plan`` (gemm_comparison.py:1419-1443)
    and, like the reference's fp32 C/D contract, writes fp32 D (beta = 0).
    """

    def __init__(self):
        self._lib = _lib.load()
        self._plan = None

    def create_plan(self, m, n, k, a_ptr, b_ptr, c_ptr, d_ptr, stream):
        if self._plan is not None:
            raise BridgeError("a plan already exists; destroy it before the next shape")
        plan = ctypes.c_void_p(None)
        info = _lib.PlanInfo()
        rc = self._lib.b200_gemm_plan_create(int(m), int(n), int(k), a_ptr, b_ptr, c_ptr, d_ptr,
                                             stream, ctypes.byref(plan), ctypes.byref(info))
        _lib.check(rc, "b200_gemm_plan_create", self._lib)
        if not plan:
            raise BridgeError("plan creation reported success but returned no plan")
        self._plan = plan
        return info

    def execute(self) -> None:
        if self._plan is None:
            raise BridgeError("no plan exists; nothing can be executed")
        _lib.check(self._lib.b200_gemm_plan_execute(self._plan), "b200_gemm_plan_execute", self._lib)

    def synchronize(self) -> None:
        if self._plan is None:
            raise BridgeError("no plan exists; nothing can be synchronized")
        _lib.check(self._lib.b200_stream_synchronize(self._plan), "b200_stream_synchronize", self._lib)

    def destroy(self) -> None:
        if self._plan is None:
            return
        plan, self._plan = self._plan, None
        _lib.check(self._lib.b200_gemm_plan_destroy(plan), "b200_gemm_plan_destroy", self._lib)


def supported(m: int, n: int, k: int, out_dtype=torch.bfloat16, mode: str = "auto",
              ldd: int | None = None) -> tuple[bool, str]:
    """Analogue of CuTe's ``can_implement``: (accepted, reason)."""
    lib = _lib.load()
    rc = lib.b200_gemm_supported(int(m), int(n), int(k), int(n if ldd is None else ldd),
                                 _DTYPE_CODE[out_dtype], _MODE_CODE[mode])
    return (rc == _lib.OK, "" if rc == _lib.OK else _lib.last_error(lib))


def gemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, *,
         out_dtype=torch.bfloat16, mode: str = "auto", stream=None):
    """D = A @ B.T through the C ABI; synchronous, checks the device status word.

    Hot loops should hold a ``GemmPlan`` and call ``execute`` instead.
    """
    m, n = a.shape[0], b.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype, device=a.device)
    plan = GemmPlan(a, b, out, mode=mode, stream=stream)
    try:
        plan.execute()
        plan.synchronize()
    finally:
        plan.destroy()
    return out


_MODE_NAME = {v: k for k, v in _MODE_CODE.items()}


def policy(m: int, n: int, k: int, *, mode: str = "auto", sm_count: int = 148) -> dict:
    """The plan's host-side choices for an M x N x K GEMM on a GPU with ``sm_count`` SMs,
    computed without a device (b200_gemm_policy): resolved mode, tile grid, raster,
    schedule (and the stream-K layout when it applies)."""
    lib = _lib.load()
    if mode not in _MODE_CODE:
        raise ValueError(f"mode must be one of {sorted(_MODE_CODE)}")
    info = _lib.PolicyInfo()
    _lib.check(lib.b200_gemm_policy(m, n, k, _MODE_CODE[mode], sm_count, ctypes.byref(info)),
               "b200_gemm_policy", lib)
    out = {name: getattr(info, name) for name, _ in info._fields_}
    out["mode"] = _MODE_NAME[out["mode"]]
    out["schedule"] = "stream_k" if out["schedule"] == 1 else "dynamic"
    return out
