#!/usr/bin/env bash
# TEST INFRASTRUCTURE ONLY. Builds oracle/_ref/libwpref.so from the
# reference's own CUDA kernel sources, where they lie in the reference
# checkout (never copied into this repository), plus oracle/ref_shim.cu.
# Usage: oracle/build_ref.sh [REFERENCE_ROOT]
# (default: $WP_REFERENCE_ROOT, else a checkout named "reference" beside
# this repository's directory)
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
REF="${1:-${WP_REFERENCE_ROOT:-$HERE/../../reference}}"
OUT="$HERE/_ref"
K="$REF/csrc/kernels"
if [ ! -f "$K/warp_pipe_r32.cu" ]; then
  echo "reference kernels not found under $K" >&2
  exit 2
fi
mkdir -p "$OUT"
NVCC="${NVCC:-nvcc}"
"$NVCC" -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -Xcompiler -fPIC -shared \
  -I "$K" -o "$OUT/libwpref.so" \
  "$HERE/ref_shim.cu" "$K/warp_pipe_r32.cu" "$K/warp_pipe_r8.cu" "$K/warp_pipe_r16.cu" "$K/warp_pipe_r64.cu"
echo "$OUT/libwpref.so"
