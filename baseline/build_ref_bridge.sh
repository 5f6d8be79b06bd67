#!/bin/sh
# Context baseline (not product): builds the reference study's own cuBLASLt
# bridge, src/gemm/cublaslt_bridge_p35.cu, unmodified, from a checkout of the
# reference repository into baseline/_ref/ (git-ignored). The drivers use it
# as the "cublaslt_p35" candidate for the reference's five frozen shapes.
# Usage: sh baseline/build_ref_bridge.sh [/path/to/reference]
set -e
REF="${1:?usage: sh baseline/build_ref_bridge.sh /path/to/reference}"
HERE="$(cd "$(dirname "$0")" && pwd)"
mkdir -p "$HERE/_ref"
nvcc -O3 -std=c++17 -shared -Xcompiler -fPIC \
    "$REF/src/gemm/cublaslt_bridge_p35.cu" -lcublasLt -o "$HERE/_ref/libcublaslt_bridge_p35.so"
echo "built $HERE/_ref/libcublaslt_bridge_p35.so"
