#!/bin/bash
# Compiles the reference's own CUDA decode kernels, unmodified, from where they
# lie in the reference checkout, for sm_100a -- TEST INFRASTRUCTURE ONLY.
# Outputs go to oracle/_ref/ (git-ignored; travels to the GPU box with the tree).
#   libref_int8.so : a10_int8_decode_kernel.cu with config.cuh prepended, as
#                    bench_int8.py:58-66 does textually (here via nvcc -include)
#   libref_bf16.so : a10_decode_kernel.cu (includes config.cuh itself)
# Flags follow bench_int8.py:262-263 / a10_decode.py:270-277 with the arch
# changed to sm_100a.  Usage: oracle/build_ref.sh [reference_dir]
# (default: $MQ_REFERENCE_DIR, else a directory named "reference" beside this repository)
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
REF="${1:-${MQ_REFERENCE_DIR:-$(dirname "$(dirname "$HERE")")/reference}}"
OUT="$HERE/_ref"
[ -f "$REF/a10_int8_decode_kernel.cu" ] || { echo "reference not found at $REF" >&2; exit 1; }
mkdir -p "$OUT"
NVCC="${CUDA_HOME:-/usr/local/cuda}/bin/nvcc"
FLAGS=(-O3 --use_fast_math -std=c++17 -gencode arch=compute_100a,code=sm_100a --expt-relaxed-constexpr
       -Xcompiler -fPIC -shared -I "$REF")
"$NVCC" "${FLAGS[@]}" -include "$REF/config.cuh" "$REF/a10_int8_decode_kernel.cu" -o "$OUT/libref_int8.so"
"$NVCC" "${FLAGS[@]}" "$REF/a10_decode_kernel.cu" -o "$OUT/libref_bf16.so"
echo "built $OUT/libref_int8.so $OUT/libref_bf16.so"
