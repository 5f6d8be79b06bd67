"""CuTe DSL context candidates: NVIDIA's Blackwell dense GEMM examples, run as they ship.

The reference's P3.5 comparison measures three CuTe DSL candidates next to
cuBLASLt (src/gemm/gemm_comparison.py:214-265, instantiated by
src/gemm/cutedsl_variants.py:1279-1347): the non-persistent `DenseGemmKernel`
(1-CTA 128x128) and the persistent `PersistentDenseGemmKernel` (1-CTA 128x128;
2-CTA 256x128, cluster 2x1), fp32 accumulation, TMA store. The reference pins
them to CUTLASS v4.6.1's example files; this image carries the CuTe DSL 4.5.0
runtime and an unpinned copy of the same example files inside the flashinfer
package, which is what runs here (loaded from that path at run time, never
copied into this repository). They are context baselines on one GPU only: the
B200 kernel never calls them, and their tensors cover this GPU's own memory.
"""
from __future__ import annotations

import importlib.util
from pathlib import Path

CANDIDATES = {
    # variant: (example file, class, mma tiler, cluster, 2-CTA instructions, persistent)
    "cutedsl_nonpersistent_1cta": ("dense_gemm.py", "DenseGemmKernel", (128, 128), (1, 1), False, False),
    "cutedsl_persistent_1cta": ("dense_gemm_persistent.py", "PersistentDenseGemmKernel", (128, 128),
                                (1, 1), False, True),
    "cutedsl_persistent_2cta": ("dense_gemm_persistent.py", "PersistentDenseGemmKernel", (256, 128),
                                (2, 1), True, True),
}

_MODULES = {}
_COMPILED = {}


def examples_dir() -> Path | None:
    """The Blackwell CuTe DSL examples vendored by flashinfer, or None."""
    spec = importlib.util.find_spec("flashinfer")
    if spec is None or not spec.submodule_search_locations:
        return None
    d = Path(list(spec.submodule_search_locations)[0]) / "data" / "cutlass" / "examples" / "python" \
        / "CuTeDSL" / "blackwell"
    return d if d.is_dir() else None


def available() -> tuple[bool, str]:
    d = examples_dir()
    if d is None:
        return False, "the flashinfer-vendored CuTe DSL examples are not installed"
    try:
        import cutlass  # noqa: F401
        import cutlass.cute  # noqa: F401
    except Exception as exc:  # noqa: BLE001
        return False, f"the CuTe DSL runtime does not import: {exc}"
    return True, str(d)


def _module(fname: str):
    if fname not in _MODULES:
        path = examples_dir() / fname
        spec = importlib.util.spec_from_file_location(f"b200_ctx_{path.stem}", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _MODULES[fname] = mod
    return _MODULES[fname]


class CuteDslPlan:
    """One compiled CuTe DSL GEMM over fixed torch tensors: D (fp32 or bf16) = A B^T."""

    def __init__(self, variant: str, a, b, out, stream):
        import time

        import cuda.bindings.driver as cuda_driver
        import cutlass
        import cutlass.cute as cute
        import cutlass.utils
        from cutlass.cute.runtime import from_dlpack

        fname, cls, tiler, cluster, two_cta, persistent = CANDIDATES[variant]
        mod = _module(fname)
        self.variant = variant
        m, k = a.shape
        n = b.shape[0]
        # The kernels' convention: A (m, k, l), B (n, k, l), C (m, n, l); K-major A and B.
        views = [t.unsqueeze(-1) for t in (a, b, out)]
        ta, tb, tc = (from_dlpack(v, assumed_align=16).mark_layout_dynamic(leading_dim=1)
                      for v in views)
        self._keep = views
        gemm = getattr(mod, cls)(cutlass.Float32, two_cta, tiler, cluster, True)
        if persistent:
            ok = gemm.can_implement((m, n, k, 1), ta.element_type, tb.element_type,
                                    tc.element_type, "k", "k", "n")
        else:
            ok = gemm.can_implement(ta, tb, tc)
        if not ok:
            raise RuntimeError(f"{variant}: the example cannot implement {m}x{n}x{k}")
        self.stream = cuda_driver.CUstream(int(stream.cuda_stream))
        self.max_active_clusters = None
        t0 = time.perf_counter()
        if persistent:
            self.max_active_clusters = cutlass.utils.HardwareInfo().get_max_active_clusters(
                cluster[0] * cluster[1])
            self.fn = cute.compile(gemm, ta, tb, tc, self.max_active_clusters, self.stream)
        else:
            self.fn = cute.compile(gemm, ta, tb, tc, self.stream)
        self.compile_ms = (time.perf_counter() - t0) * 1e3
        self.args = (ta, tb, tc, self.stream)
        self.meta = {"scheduler": "static_persistent" if persistent else "nonpersistent",
                     "mma_tiler_m": tiler[0], "mma_tiler_n": tiler[1], "cluster_m": cluster[0],
                     "cluster_n": cluster[1], "use_2cta_instrs": two_cta, "use_tma_store": True,
                     "max_active_clusters": self.max_active_clusters,
                     "compile_time_ms": self.compile_ms,
                     "upstream_kernel_file": f"flashinfer/data/cutlass/examples/python/CuTeDSL/blackwell/{fname}"}
        self.source = examples_dir() / fname

    def execute(self):
        self.fn(*self.args)

    def synchronize(self):
        import torch
        torch.cuda.synchronize()

    def destroy(self):
        self.fn = None
        self._keep = None
