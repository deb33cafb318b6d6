#!/bin/bash
# Builds the reference's model code against libb2g.so through the drop-in cublas_ops.cuh,
# without modifying the reference tree: a build directory gets symlinks to the reference's
# sources, its cublas_ops.cuh as cublas_ops_cublaslt.cuh, and the drop-in as cublas_ops.cuh.
#
#   build_reference_with_b2g.sh <reference_dir> <build_dir> [translation_unit.cu]
#
# The default translation unit is ab_check.cu (includes chroma.cuh, t5.cuh, attention.cuh
# and compares every routed entry point with the original cuBLASLt code).  Produces
# <build_dir>/ab_check.  Needs the cudnn-frontend headers the reference itself needs.
set -euo pipefail
REF=${1:?reference dir}
OUT=${2:?build dir}
HERE=$(cd "$(dirname "$0")" && pwd)
PKG=$(dirname "$HERE")
REPO=$(dirname "$PKG")
TU=${3:-$HERE/ab_check.cu}
NVCC=${NVCC:-/usr/local/cuda/bin/nvcc}
SITE=$(python3 -c 'import sysconfig; print(sysconfig.get_paths()["purelib"])')
mkdir -p "$OUT"
SRC=$(mktemp -d)
trap 'rm -rf "$SRC"' EXIT
for f in "$REF"/*.cuh "$REF"/*.cu "$REF"/*.h; do
  b=$(basename "$f")
  [ "$b" = "cublas_ops.cuh" ] && continue
  ln -sf "$f" "$SRC/$b"
done
ln -sf "$REF/cublas_ops.cuh" "$SRC/cublas_ops_cublaslt.cuh"
ln -sf "$HERE/cublas_ops.cuh" "$SRC/cublas_ops.cuh"
ln -sf "$TU" "$SRC/$(basename "$TU")"
"$NVCC" -gencode arch=compute_100a,code=sm_100a -O1 -std=c++17 --expt-relaxed-constexpr --extended-lambda \
  -I"$SRC" -I"$REPO/include" -I"$SITE/include" -w \
  "$SRC/$(basename "$TU")" -o "$OUT/$(basename "$TU" .cu)" \
  -L"$PKG/lib" -lb2g -Xlinker -rpath="$PKG/lib" -lcublas -lcublasLt -L"$SITE/nvidia/cudnn/lib" -l:libcudnn.so.9 \
  -Xlinker -rpath="$SITE/nvidia/cudnn/lib"
echo "$OUT/$(basename "$TU" .cu)"
