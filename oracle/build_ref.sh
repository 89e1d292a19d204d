#!/usr/bin/env bash
# Builds the reference's own CUDA kernels, unchanged, from their sources under the reference checkout into
# oracle/_ref/<op>/libkernel.so (and oracle/_ref/softmax_seed/libkernel.so), for sm_100a, with the same nvcc line
# as this repository's libraries. These are the reference implementation run on a B200 to pin the oracle
# (tests/golden/make_golden.py --gpu) and to time the reference's kernels beside this repository's; they are test
# infrastructure. oracle/_ref/ is git-ignored (built artefacts) but travels to the GPU box with the tree.
# Usage: oracle/build_ref.sh <reference_root>   (the reference checkout; a missing root is not an error)
set -euo pipefail
REF="${1:-}"
if [ -z "$REF" ]; then
  echo "build_ref: no reference root given; skipped"
  exit 0
fi
HERE="$(cd "$(dirname "$0")" && pwd)"
OUT="$HERE/_ref"
NVCC="${CUDA_HOME:-/usr/local/cuda}/bin/nvcc"
FLAGS=(-gencode arch=compute_100a,code=sm_100a -lineinfo -O3 -std=c++17 -shared -Xcompiler -fPIC)
if [ ! -d "$REF" ]; then
  echo "build_ref: no reference at $REF; skipped"
  exit 0
fi
build() {  # build <name> <source>
  mkdir -p "$OUT/$1"
  if [ ! -f "$OUT/$1/libkernel.so" ] || [ "$2" -nt "$OUT/$1/libkernel.so" ]; then
    "$NVCC" "${FLAGS[@]}" -o "$OUT/$1/libkernel.so" "$2"
  fi
}
build softmax "$REF/softmax/kernel.cu" &
build softmax_seed "$REF/softmax/seed.cu" &
build rmsnorm "$REF/rmsnorm/kernel.cu" &
build rope "$REF/rope/kernel.cu" &
build topk "$REF/topk/kernel.cu" &
wait
echo "build_ref: $(ls "$OUT")"
