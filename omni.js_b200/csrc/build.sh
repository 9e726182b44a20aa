#!/usr/bin/env bash
# Builds libminisample.so (sm_100a) in-tree next to the Python host package.
#   bash omni.js_b200/csrc/build.sh
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
OUT="$HERE/../minisample/libminisample.so"
NVCC="${NVCC:-nvcc}"
"$NVCC" -O3 -std=c++17 -gencode arch=compute_100a,code=sm_100a -lineinfo \
  -Xcompiler -fPIC -Xcompiler -Wall -shared \
  ${MS_NVCC_EXTRA:-} \
  "$HERE/ms_kernels.cu" "$HERE/ms_api.cu" -o "$OUT" -lcudart
echo "$OUT"
