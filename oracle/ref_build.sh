#!/usr/bin/env bash
# Builds oracle/_ref/libgpl_ref.so from the reference runner's own sources
# where they lie (read-only tree; nothing is copied). TEST INFRASTRUCTURE:
# the parity tests use it to pin the oracle against the reference itself.
#   gemm_lt.cu        cuBLASLt FP8 GEMM wrapper (gpl_lt_init/enqueue/free)
#   workload_util.c   work accounting
#   args.c            gpl_args_defaults / gpl_prec_name
#   util.c            logging helpers
#   ref_shim.cu       includes workload_memstream.cu and workload_powervirus.cu
#   ref_gemm_shim.c   includes workload_gemm.c (the cublasGemmEx GEMM rung)
# Usage: oracle/ref_build.sh [REFERENCE_ROOT]   (default /root/reference)
set -euo pipefail
REF=${1:-/root/reference}
SRC="$REF/runner/src"
HERE="$(cd "$(dirname "$0")" && pwd)"
OUT="$HERE/_ref"
if [ ! -d "$SRC" ]; then
    echo "ref_build: $SRC not found; skipping" >&2
    exit 0
fi
mkdir -p "$OUT"
TMP="$(mktemp -d)"
trap 'rm -rf "$TMP"' EXIT
GEN="-gencode arch=compute_100a,code=sm_100a"
gcc -std=gnu11 -O2 -fPIC -I"$SRC" -I/usr/local/cuda/include -c "$SRC/args.c" -o "$TMP/args.o"
gcc -std=gnu11 -O2 -fPIC -I"$SRC" -I/usr/local/cuda/include -c "$SRC/util.c" -o "$TMP/util.o"
gcc -std=gnu11 -O2 -fPIC -I"$SRC" -I/usr/local/cuda/include -c "$SRC/workload_util.c" -o "$TMP/workload_util.o"
nvcc $GEN -O2 -Xcompiler -fPIC -I"$SRC" -c "$SRC/gemm_lt.cu" -o "$TMP/gemm_lt.o"
nvcc $GEN -O2 -Xcompiler -fPIC -I"$SRC" -c "$HERE/ref_shim.cu" -o "$TMP/ref_shim.o"
gcc -std=gnu11 -O2 -fPIC -I"$SRC" -I/usr/local/cuda/include -c "$HERE/ref_gemm_shim.c" -o "$TMP/ref_gemm_shim.o"
nvcc $GEN -shared -o "$OUT/libgpl_ref.so" "$TMP"/*.o -lcublasLt -lcublas
# Record where the reference tree was found, for the tests that read its
# schema and host sources (they skip where this file names no tree).
printf '%s\n' "$REF" > "$OUT/reference_root"
echo "ref_build: wrote $OUT/libgpl_ref.so"
