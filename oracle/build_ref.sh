#!/bin/sh
# Builds the reference's own CUDA hot path (cuda_kernels.cu, transformer.cu,
# sageattention_sm80.cu via ref_harness.cu) from the reference tree, with the
# reference Makefile's flags (its Makefile:11) for sm_100a, into
# oracle/_ref/libqiref.so.  Test infrastructure: the parity checker and the
# reference arm of bench.py.  main.cu is not built (it needs libpng).
set -e
REF=${QI_REFERENCE_DIR:-/root/reference}
HERE=$(cd "$(dirname "$0")" && pwd)
OUT="$HERE/_ref"
if [ ! -f "$REF/transformer.cu" ]; then
  echo "reference sources not found at $REF; skipping oracle/_ref" >&2
  exit 0
fi
mkdir -p "$OUT"
NVCC=${NVCC:-/usr/local/cuda/bin/nvcc}
FLAGS="-O2 -std=c++17 --expt-relaxed-constexpr --extended-lambda -diag-suppress=177 --use_fast_math"
ARCH="-gencode arch=compute_100a,code=sm_100a"
for src in cuda_kernels transformer; do
  "$NVCC" $FLAGS $ARCH -I"$REF" -Xcompiler -fPIC -ccbin g++ -c "$REF/$src.cu" -o "$OUT/$src.o" &
done
"$NVCC" $FLAGS $ARCH -I"$REF" -Xcompiler -fPIC -ccbin g++ -c "$HERE/ref_harness.cu" -o "$OUT/ref_harness.o" &
wait
"$NVCC" $ARCH -shared -ccbin g++ -o "$OUT/libqiref.so" "$OUT/cuda_kernels.o" "$OUT/transformer.o" \
  "$OUT/ref_harness.o" -lcublas -lcusolver
echo "built $OUT/libqiref.so"
