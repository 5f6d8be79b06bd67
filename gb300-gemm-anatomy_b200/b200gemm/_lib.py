"""ctypes binding of ``libb200gemm.so`` (declared in ``include/b200gemm.h``).

The loader mirrors the reference driver's bridge front end
(``src/gemm/gemm_comparison.py:1299-1460``): it checks the ABI version and the
byte size of every metadata struct against these ctypes mirrors, turns every
non-zero return code into an exception carrying the library's own thread-local
diagnostic, and never retries or falls back. There is no CPU path: if the
shared library is missing the import of the GPU entry points fails loudly.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

ABI_VERSION = 1

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_DEVICE_TIMEOUT = 4
ERR_MISMATCH = 5
ERR_NO_DEVICE = 6
ERR_INTERNAL = 7

OUT_BF16 = 0
OUT_F32 = 1

MODE_AUTO = 0
MODE_1CTA = 1
MODE_2CTA = 2
MODE_2CTA_M512 = 3
MODE_2CTA_N128 = 4

STREAM_LDGSTS = 0
STREAM_TMA = 1
STREAM_TMA_SW128 = 2

STREAM_VALIDATE = 0
STREAM_CHECKSUM = 1
STREAM_SINK = 2

DEV_STATUS_NAMES = {
    0x101: "TIMEOUT_PRODUCER",
    0x102: "TIMEOUT_MMA_FULL",
    0x103: "TIMEOUT_MMA_TMEM",
    0x104: "TIMEOUT_EPILOGUE",
    0x105: "TIMEOUT_STREAM",
    0x106: "TIMEOUT_UMMA",
    0x107: "TIMEOUT_SELFTEST",
    0x108: "TIMEOUT_PARTIAL",
    0x1FF: "BAD_LAUNCH",
}

LIB_NAME = "libb200gemm.so"
LIB_PATH = Path(os.environ.get("B200GEMM_LIB", Path(__file__).resolve().parent / LIB_NAME))


class BridgeError(RuntimeError):
    """A C-ABI call returned a non-zero status (message from b200_last_error)."""

    def __init__(self, message: str, code: int = ERR_INTERNAL):
        super().__init__(message)
        self.code = code


class CorrectnessError(RuntimeError):
    """A result failed its parity check against the oracle."""


def _i64_struct(name, fields, doubles=()):
    members = [(f, ctypes.c_int64) for f in fields] + [(f, ctypes.c_double) for f in doubles]
    return type(name, (ctypes.Structure,), {"_fields_": members})


DeviceInfo = _i64_struct(
    "B200DeviceInfo",
    ["device", "cc_major", "cc_minor", "sm_count", "l2_bytes", "smem_per_sm_bytes",
     "smem_optin_bytes", "global_mem_bytes", "driver_version", "runtime_version",
     "clock_khz", "is_sm100"],
)

PlanInfo = _i64_struct(
    "B200PlanInfo",
    ["abi_version", "m", "n", "k", "lda", "ldb", "ldd", "out_dtype", "mode", "cta_group",
     "tile_m", "tile_n", "tile_k", "stages", "cluster_m", "grid_ctas", "threads_per_cta",
     "smem_bytes", "tmem_columns", "num_tiles", "sm_count", "device"],
    doubles=["waves", "flop_count"],
)

PolicyInfo = _i64_struct(
    "B200PolicyInfo",
    ["mode", "tile_m", "tile_n", "num_m_blocks", "num_n_blocks", "num_k_blocks", "num_tiles",
     "clusters", "raster_n", "group", "schedule", "sk_groups", "sk_lanes", "sk_lane_n",
     "sk_rounds", "sk_split_tiles", "grid_ctas", "kserp_wave"],
    doubles=["waves"],
)

StreamConfig = _i64_struct(
    "B200StreamConfig", ["method", "stages", "stage_bytes", "ctas_per_sm", "passes", "rotation"]
)

StreamResult = _i64_struct(
    "B200StreamResult",
    ["grid_ctas", "threads_per_cta", "smem_bytes", "occupancy_ctas_per_sm", "tiles_per_cta",
     "bytes_streamed", "mismatches", "checksum_xor", "checksum_sum", "sink_xor", "status"],
)

UmmaConfig = _i64_struct(
    "B200UmmaConfig", ["cta_group", "n", "depth", "iterations", "timed", "num_ctas"]
)

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_INT = ctypes.c_int

# name -> (restype, argtypes); every symbol declared in include/b200gemm.h.
SIGNATURES = {
    "b200_abi_version": (_INT, []),
    "b200_plan_info_size": (ctypes.c_size_t, []),
    "b200_device_info_size": (ctypes.c_size_t, []),
    "b200_stream_result_size": (ctypes.c_size_t, []),
    "b200_last_error": (ctypes.c_char_p, []),
    "b200_device_probe": (_INT, [_INT, ctypes.POINTER(DeviceInfo)]),
    "b200_gemm_plan_create": (_INT, [_I64, _I64, _I64, _P, _P, _P, _P, _P,
                                     ctypes.POINTER(_P), ctypes.POINTER(PlanInfo)]),
    "b200_gemm_plan_create_ex": (_INT, [_I64, _I64, _I64, _P, _P, _P, _I64, _INT, _INT, _P,
                                        ctypes.POINTER(_P), ctypes.POINTER(PlanInfo)]),
    "b200_gemm_plan_execute": (_INT, [_P]),
    "b200_gemm_plan_execute_on": (_INT, [_P, _P]),
    "b200_stream_synchronize": (_INT, [_P]),
    "b200_gemm_plan_destroy": (_INT, [_P]),
    "b200_gemm_supported": (_INT, [_I64, _I64, _I64, _I64, _INT, _INT]),
    "b200_gemm": (_INT, [_I64, _I64, _I64, _P, _P, _P, _I64, _INT, _INT, _P]),
    "b200_gemm_plan_launches": (_I64, [_P]),
    "b200_gemm_plan_schedule": (_INT, [_P]),
    "b200_policy_info_size": (ctypes.c_size_t, []),
    "b200_gemm_policy": (_INT, [_I64, _I64, _I64, _INT, _INT, ctypes.POINTER(PolicyInfo)]),
    "b200_gemm_plan_set_trace": (_INT, [_P, _P, _I64]),
    "b200_gemm_plan_set_peers": (_INT, [_P, _INT, ctypes.POINTER(_P)]),
    "b200_gemm_plan_set_multicast": (_INT, [_P, _P]),
    "b200_ipc_handle_size": (ctypes.c_size_t, []),
    "b200_peer_buffer_alloc": (_INT, [_I64, ctypes.POINTER(_P), _P]),
    "b200_peer_buffer_free": (_INT, [_P]),
    "b200_peer_open": (_INT, [_P, ctypes.POINTER(_P)]),
    "b200_peer_close": (_INT, [_P]),
    "b200_peer_copy_2d": (_INT, [_P, _I64, _P, _I64, _I64, _I64, _P]),
    "b200_gemm_noalloc": (_INT, [_I64, _I64, _I64, _P, _P, _P, _I64, _INT, _INT, _P]),
    "b200_fill_pattern": (_INT, [_P, _I64, _P]),
    "b200_stream_plan_create": (_INT, [ctypes.POINTER(StreamConfig), _P, _I64, _INT,
                                       ctypes.POINTER(_P), ctypes.POINTER(StreamResult)]),
    "b200_stream_plan_granule": (_I64, [ctypes.POINTER(StreamConfig), _INT]),
    "b200_stream_plan_execute": (_INT, [_P, _INT, _P]),
    "b200_stream_plan_result": (_INT, [_P, _P, ctypes.POINTER(StreamResult)]),
    "b200_stream_plan_destroy": (_INT, [_P]),
    "b200_umma_probe": (_INT, [ctypes.POINTER(UmmaConfig), _P, _P, _P, _P, _P, _P]),
    "b200_selftest_bounded_wait": (_INT, [ctypes.c_ulonglong, _P, _P]),
    "b200_selftest_occupy": (_INT, [_INT, _INT, ctypes.c_ulonglong, _P]),
    "b200_shard_range": (_INT, [_I64, _I64, _I64, _I64, ctypes.POINTER(_I64),
                                ctypes.POINTER(_I64)]),
}

_STRUCT_SIZES = {
    "b200_plan_info_size": PlanInfo,
    "b200_device_info_size": DeviceInfo,
    "b200_stream_result_size": StreamResult,
    "b200_policy_info_size": PolicyInfo,
}

_lib = None


def load(path: Path | None = None):
    """Load and handshake the shared library once; raise BridgeError on any mismatch."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    lib_path = Path(path) if path is not None else LIB_PATH
    if not lib_path.is_file():
        raise BridgeError(
            f"{lib_path} is missing: build it with `make -C gb300-gemm-anatomy_b200/csrc` "
            "(or __graft_entry__.build()); there is no fallback path",
            ERR_INTERNAL,
        )
    try:
        lib = ctypes.CDLL(str(lib_path))
    except OSError as exc:
        raise BridgeError(f"cannot load {lib_path}: {exc}") from exc
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    abi = int(lib.b200_abi_version())
    if abi != ABI_VERSION:
        raise BridgeError(f"{lib_path} reports ABI version {abi}, this binding expects {ABI_VERSION}")
    for fn_name, struct in _STRUCT_SIZES.items():
        size = int(getattr(lib, fn_name)())
        if size != ctypes.sizeof(struct):
            raise BridgeError(
                f"{fn_name} reports {size} bytes, the ctypes mirror {struct.__name__} has "
                f"{ctypes.sizeof(struct)}; the ABI does not match"
            )
    if path is None:
        _lib = lib
    return lib


def last_error(lib=None) -> str:
    lib = lib or load()
    raw = lib.b200_last_error()
    return raw.decode("utf-8", errors="replace") if raw else "no diagnostic"


def check(rc: int, what: str, lib=None) -> None:
    if rc != OK:
        raise BridgeError(f"{what} failed (code {rc}): {last_error(lib)}", rc)


def shard_range(n: int, world: int, rank: int, granule: int = 16):
    """[begin, end) output columns of shard `rank` (C-ABI b200_shard_range)."""
    lib = load()
    b = _I64(0)
    e = _I64(0)
    check(lib.b200_shard_range(n, world, rank, granule, ctypes.byref(b), ctypes.byref(e)),
          "b200_shard_range", lib)
    return int(b.value), int(e.value)


def device_probe(device: int = 0):
    lib = load()
    info = DeviceInfo()
    check(lib.b200_device_probe(device, ctypes.byref(info)), "b200_device_probe", lib)
    return {name: getattr(info, name) for name, _ in DeviceInfo._fields_}
