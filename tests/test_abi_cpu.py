"""C-ABI boundary on the CPU: the library loads, exports every declared symbol,
passes the size/version handshake and validates arguments without a GPU."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from b200gemm import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "b200gemm.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b200_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_and_library_exports_every_symbol():
    names = declared_functions()
    assert len(names) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (b200_\w+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    # the ctypes binding covers exactly the header
    assert sorted(_lib.SIGNATURES) == names


def test_handshake():
    lib = _lib.load()
    assert lib.b200_abi_version() == _lib.ABI_VERSION
    assert lib.b200_plan_info_size() == ctypes.sizeof(_lib.PlanInfo)
    assert lib.b200_device_info_size() == ctypes.sizeof(_lib.DeviceInfo)
    assert lib.b200_stream_result_size() == ctypes.sizeof(_lib.StreamResult)


def test_supported_rules():
    lib = _lib.load()
    f = lib.b200_gemm_supported
    assert f(8192, 8192, 8192, 8192, _lib.OUT_BF16, _lib.MODE_AUTO) == _lib.OK
    assert f(512, 128256 // 8, 4096, 128256 // 8, _lib.OUT_BF16, _lib.MODE_2CTA) == _lib.OK
    assert f(64, 64, 60, 64, _lib.OUT_BF16, 0) == _lib.ERR_UNSUPPORTED  # K % 8
    assert "K %" in _lib.last_error(lib) or "16-byte" in _lib.last_error(lib)
    assert f(64, 64, 64, 32, _lib.OUT_BF16, 0) == _lib.ERR_INVALID_ARGUMENT  # ldd < n
    assert f(64, 257, 64, 257, _lib.OUT_BF16, 0) == _lib.ERR_UNSUPPORTED  # pitch % 16
    assert f(64, 257, 64, 260, _lib.OUT_F32, 0) == _lib.OK
    assert f(64, 64, 64, 64, 7, 0) == _lib.ERR_INVALID_ARGUMENT
    assert f(64, 64, 64, 64, 0, 9) == _lib.ERR_INVALID_ARGUMENT
    assert f(-1, 64, 64, 64, 0, 0) == _lib.ERR_INVALID_ARGUMENT
    assert f(1 << 31, 64, 64, 64, 0, 0) == _lib.ERR_UNSUPPORTED


def test_plan_create_rejects_bad_arguments_without_gpu():
    lib = _lib.load()
    plan = ctypes.c_void_p()
    info = _lib.PlanInfo()
    rc = lib.b200_gemm_plan_create_ex(64, 64, 64, None, None, None, 64, 0, 0, None,
                                      ctypes.byref(plan), ctypes.byref(info))
    assert rc == _lib.ERR_INVALID_ARGUMENT and not plan
    rc = lib.b200_gemm_plan_create_ex(64, 64, 64, 8, 16, 32, 64, 0, 0, None, None, None)
    assert rc == _lib.ERR_INVALID_ARGUMENT
    assert lib.b200_gemm_plan_destroy(None) == _lib.OK
    assert lib.b200_gemm_plan_execute(None) == _lib.ERR_INVALID_ARGUMENT


def test_device_probe_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    lib = _lib.load()
    info = _lib.DeviceInfo()
    assert lib.b200_device_probe(0, ctypes.byref(info)) == _lib.ERR_NO_DEVICE


def test_stream_config_validation():
    lib = _lib.load()
    cfg = _lib.StreamConfig(_lib.STREAM_LDGSTS, 3, 8192, 1, 1, 0)
    assert lib.b200_stream_plan_granule(ctypes.byref(cfg), 0) == -1
    cfg = _lib.StreamConfig(_lib.STREAM_TMA, 4, 16384, 2, 1, 0)
    assert lib.b200_stream_plan_granule(ctypes.byref(cfg), 0) == 16384
    plan = ctypes.c_void_p()
    cfg = _lib.StreamConfig(_lib.STREAM_LDGSTS, 4, 3000, 1, 1, 0)
    assert lib.b200_stream_plan_create(ctypes.byref(cfg), 1024, 1 << 20, 0, ctypes.byref(plan),
                                       None) == _lib.ERR_INVALID_ARGUMENT


def test_umma_config_validation():
    lib = _lib.load()
    cfg = _lib.UmmaConfig(1, 96, 4, 1, 0, 0)
    assert lib.b200_umma_probe(ctypes.byref(cfg), None, None, 16, None, 32, None) == \
        _lib.ERR_INVALID_ARGUMENT
    cfg = _lib.UmmaConfig(3, 64, 4, 1, 0, 0)
    assert lib.b200_umma_probe(ctypes.byref(cfg), None, None, 16, None, 32, None) == \
        _lib.ERR_INVALID_ARGUMENT
    cfg = _lib.UmmaConfig(1, 64, 5, 1, 0, 0)
    assert lib.b200_umma_probe(ctypes.byref(cfg), None, None, 16, None, 32, None) == \
        _lib.ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("n,world,granule", [(128256, 8, 16), (4096, 2, 16), (14336, 4, 16),
                                             (100, 3, 16), (8, 8, 16), (0, 2, 16)])
def test_shard_range_partitions(n, world, granule):
    ranges = [_lib.shard_range(n, world, r, granule) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (b0, e0), (b1, e1) in zip(ranges, ranges[1:]):
        assert e0 == b1
    for b, e in ranges:
        assert b <= e and (b % granule == 0 or b == n)
    assert _lib.shard_range(128256, 8, 0, 16) == (0, 16032)


_C_CALLER = r"""
#include <stdio.h>
#include "b200gemm.h"

int main(void) {
    B200Plan* plan = NULL;
    if (b200_abi_version() != B200_ABI_VERSION) return 1;
    if (b200_plan_info_size() != sizeof(B200PlanInfo)) return 2;
    if (b200_gemm_supported(8192, 8192, 8192, 8192, B200_OUT_BF16, B200_MODE_AUTO) != B200_OK) return 3;
    if (b200_gemm_supported(64, 64, 60, 64, B200_OUT_BF16, B200_MODE_AUTO) != B200_ERR_UNSUPPORTED) return 4;
    if (b200_gemm_plan_schedule(NULL) != -1) return 5;
    if (b200_gemm_plan_create_ex(64, 64, 64, NULL, NULL, NULL, 64, B200_OUT_BF16, B200_MODE_AUTO,
                                 NULL, &plan, NULL) != B200_ERR_INVALID_ARGUMENT) return 6;
    if (plan != NULL) return 7;
    printf("%s\n", b200_last_error());
    return 0;
}
"""


def test_header_is_plain_c_and_links(tmp_path):
    """A C99 caller compiles against include/b200gemm.h with warnings as errors, links
    against the library and gets the handshake and argument checks without a GPU."""
    src = tmp_path / "caller.c"
    src.write_text(_C_CALLER)
    exe = tmp_path / "caller"
    libdir = _lib.LIB_PATH.parent
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-I", str(HEADER.parent),
                    str(src), "-o", str(exe), f"-L{libdir}", "-l:" + _lib.LIB_PATH.name,
                    f"-Wl,-rpath,{libdir}"], check=True, capture_output=True, text=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert res.returncode == 0, (res.returncode, res.stdout, res.stderr)
    assert "device pointer" in res.stdout  # the thread-local message of the last failed call
