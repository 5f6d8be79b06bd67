"""b200gemm: B200-native (sm_100a) BF16 GEMM stack behind the GB300 GEMM-anatomy driver API.

Layers: memory-path streamers (LDGSTS / TMA), a persistent warp-specialised
tcgen05 GEMM (1-CTA and 2-CTA), and N-sharding over several GPUs. All compute
runs in ``libb200gemm.so`` through the C ABI in ``include/b200gemm.h``.
"""
from ._lib import BridgeError, CorrectnessError, load, device_probe, shard_range  # noqa: F401

__all__ = ["BridgeError", "CorrectnessError", "load", "device_probe", "shard_range"]
__version__ = "0.1.0"
