#!/usr/bin/env bash
# Builds two runner binaries from the reference tree where it lies (nothing
# is copied), into oracle/_ref/:
#   gpu-power-runner        the unmodified reference runner (all of
#                           runner/src), for same-box comparisons
#   gpu-power-runner-gplk   the reference's kept host (main, args, telemetry,
#                           probe, util, fft, observe, nccl) with this
#                           repository's drop-ins for the load generators and
#                           the summary emitter (gpu-power-lab_b200/runner/
#                           *.c|cu, include/gemm_lt.h) linked to libgplk.so
# TEST INFRASTRUCTURE: the integration tests run both. Neither binary
# touches power limits or clocks unless given --power-limit,
# --raise-power-limit or --lock-clocks, which the tests never pass.
# Usage: oracle/runner_build.sh [REFERENCE_ROOT]   (default /root/reference)
set -euo pipefail
REF=${1:-/root/reference}
SRC="$REF/runner/src"
HERE="$(cd "$(dirname "$0")" && pwd)"
REPO="$(cd "$HERE/.." && pwd)"
OUT="$HERE/_ref"
DROP="$REPO/gpu-power-lab_b200/runner"
if [ ! -d "$SRC" ]; then
    echo "runner_build: $SRC not found; skipping" >&2
    exit 0
fi
mkdir -p "$OUT"
TMP="$(mktemp -d)"
trap 'rm -rf "$TMP"' EXIT
CUDA=/usr/local/cuda
GEN="-gencode arch=compute_100a,code=sm_100a"
CFLAGS="-std=gnu11 -O2 -Wall -Wno-unused-parameter -DGPL_HAVE_NCCL -I$CUDA/include"
NVFLAGS="$GEN -O3 -std=c++17 -DGPL_HAVE_NCCL"
LIBS="-L$CUDA/lib64 -L$CUDA/lib64/stubs -lcublas -lcublasLt -lcufft -lnvidia-ml -lnccl -lpthread -lm"
KEPT_C="main.c args.c telemetry.c probe.c workload_observe.c workload_fft.c util.c"

# 1. the reference as it is
mkdir -p "$TMP/ref"
for f in $KEPT_C summary.c workload_gemm.c workload_util.c; do
    gcc $CFLAGS -I"$SRC" -c "$SRC/$f" -o "$TMP/ref/${f%.c}.o"
done
for f in workload_memstream.cu workload_powervirus.cu gemm_lt.cu workload_nccl.cu; do
    nvcc $NVFLAGS -I"$SRC" -c "$SRC/$f" -o "$TMP/ref/${f%.cu}.o"
done
nvcc $GEN -o "$OUT/gpu-power-runner" "$TMP"/ref/*.o $LIBS

# 2. kept host + drop-ins + libgplk.so (this tree's include/ shadows gemm_lt.h)
mkdir -p "$TMP/gplk"
INC="-I$REPO/include -I$DROP -I$SRC"
for f in $KEPT_C; do
    gcc $CFLAGS -I"$SRC" -c "$SRC/$f" -o "$TMP/gplk/${f%.c}.o"
done
nvcc $NVFLAGS -I"$SRC" -c "$SRC/workload_nccl.cu" -o "$TMP/gplk/workload_nccl.o"
for f in workload_gemm.c workload_util.c summary.c; do
    gcc $CFLAGS $INC -c "$DROP/$f" -o "$TMP/gplk/drop_${f%.c}.o"
done
for f in workload_memstream.cu workload_powervirus.cu fabric_step.cu; do
    nvcc $NVFLAGS $INC -c "$DROP/$f" -o "$TMP/gplk/drop_${f%.cu}.o"
done
nvcc $GEN -o "$OUT/gpu-power-runner-gplk" "$TMP"/gplk/*.o \
    -L"$REPO/gpu-power-lab_b200" -lgplk -Xlinker -rpath -Xlinker '$ORIGIN/../../gpu-power-lab_b200' $LIBS
echo "runner_build: wrote $OUT/gpu-power-runner and $OUT/gpu-power-runner-gplk"
