#!/bin/bash
# Builds the reference's model code against libb2g.so through the drop-in headers, without
# modifying the reference tree: a build directory gets symlinks to the reference's sources,
# its three routed headers under new names (cublas_ops.cuh as cublas_ops_cublaslt.cuh,
# cudnn_attention.cuh as cudnn_attention_cudnn.cuh, attention.cuh as attention_cublas.cuh)
# and the drop-ins (this directory) under the original names.
#
#   build_reference_with_b2g.sh <reference_dir> <build_dir> [translation_unit.cu] [--shared]
#
# The default translation unit is ab_check.cu (includes chroma.cuh, t5.cuh, attention.cuh
# and compares every routed entry point with the original code).  Produces
# <build_dir>/<unit> (an executable), or <build_dir>/lib<unit>_b2g.so with --shared.  Needs
# the cudnn-frontend headers the reference itself needs.
set -euo pipefail
REF=${1:?reference dir}
OUT=${2:?build dir}
HERE=$(cd "$(dirname "$0")" && pwd)
PKG=$(dirname "$HERE")
REPO=$(dirname "$PKG")
TU=${3:-$HERE/ab_check.cu}
SHARED=${4:-}
NVCC=${NVCC:-/usr/local/cuda/bin/nvcc}
SITE=$(python3 -c 'import sysconfig; print(sysconfig.get_paths()["purelib"])')
mkdir -p "$OUT"
SRC=$(mktemp -d)
trap 'rm -rf "$SRC"' EXIT
for f in "$REF"/*.cuh "$REF"/*.cu "$REF"/*.h; do
  b=$(basename "$f")
  case "$b" in cublas_ops.cuh|cudnn_attention.cuh|attention.cuh) continue ;; esac
  ln -sf "$f" "$SRC/$b"
done
ln -sf "$REF/cublas_ops.cuh" "$SRC/cublas_ops_cublaslt.cuh"
ln -sf "$REF/cudnn_attention.cuh" "$SRC/cudnn_attention_cudnn.cuh"
ln -sf "$REF/attention.cuh" "$SRC/attention_cublas.cuh"
for h in cublas_ops.cuh cudnn_attention.cuh attention.cuh; do ln -sf "$HERE/$h" "$SRC/$h"; done
ln -sf "$TU" "$SRC/$(basename "$TU")"
NAME=$(basename "$TU" .cu)
if [ "$SHARED" = "--shared" ]; then
  TARGET="$OUT/lib${NAME}_b2g.so"
  KIND=(-shared -Xcompiler -fPIC -Xlinker -Bsymbolic)
else
  TARGET="$OUT/$NAME"
  KIND=()
fi
# -O3 --use_fast_math: the reference's own flags (its CMakeLists.txt), so that the kernels the
# drop-in build keeps (elementwise, RoPE producers) compute exactly as in the stock build.
"$NVCC" -gencode arch=compute_100a,code=sm_100a -O3 --use_fast_math -std=c++17 --expt-relaxed-constexpr \
  --extended-lambda "${KIND[@]}" -I"$SRC" -I"$REPO/include" -I"$SITE/include" -w \
  "$SRC/$(basename "$TU")" -o "$TARGET" \
  -L"$PKG/lib" -lb2g -Xlinker -rpath="$PKG/lib" -lcublas -lcublasLt -L"$SITE/nvidia/cudnn/lib" -l:libcudnn.so.9 \
  -Xlinker -rpath="$SITE/nvidia/cudnn/lib"
echo "$TARGET"
