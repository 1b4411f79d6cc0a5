#!/bin/sh
# Builds the reference's own CUDA hot path from the reference tree (cuda_kernels.cu,
# transformer.cu, and sageattention_sm80.cu included by ref_harness.cu) with the
# reference Makefile's flags (its Makefile:11) for sm_100a:
#   oracle/_ref/libqiref.so     reference ops + transformer_forward (parity checker,
#                               reference arm of bench.py)
#   oracle/_ref/libshimtest.so  the same caller code (ref_driver.cu) linked against the
#                               product's drop-in shim instead of transformer.cu
# Test infrastructure.  main.cu is not built (it needs libpng).
set -e
REF=${QI_REFERENCE_DIR:?set QI_REFERENCE_DIR to the reference source tree}
HERE=$(cd "$(dirname "$0")" && pwd)
PKG="$HERE/../qwen-image.cu_b200"
OUT="$HERE/_ref"
if [ ! -f "$REF/transformer.cu" ]; then
  echo "reference sources not found at $REF; skipping oracle/_ref" >&2
  exit 0
fi
mkdir -p "$OUT"
NVCC=${NVCC:-/usr/local/cuda/bin/nvcc}
FLAGS="-O2 -std=c++17 --expt-relaxed-constexpr --extended-lambda -diag-suppress=177 --use_fast_math"
ARCH="-gencode arch=compute_100a,code=sm_100a"
CC="$NVCC $FLAGS $ARCH -I$REF -I$HERE/../include -Xcompiler -fPIC -ccbin g++"
$CC -c "$REF/cuda_kernels.cu" -o "$OUT/cuda_kernels.o" &
$CC -c "$REF/transformer.cu" -o "$OUT/transformer.o" &
$CC -c "$HERE/ref_harness.cu" -o "$OUT/ref_harness.o" &
$CC -c "$HERE/ref_driver.cu" -o "$OUT/ref_driver.o" &
$CC -x cu -c "$PKG/shim/transformer_b200.cpp" -o "$OUT/transformer_b200.o" &
wait
for o in cuda_kernels transformer ref_harness ref_driver transformer_b200; do
  [ -f "$OUT/$o.o" ] || { echo "compile of $o failed" >&2; exit 1; }
done
"$NVCC" $ARCH -shared -ccbin g++ -o "$OUT/libqiref.so" "$OUT/cuda_kernels.o" "$OUT/transformer.o" \
  "$OUT/ref_harness.o" "$OUT/ref_driver.o" -lcublas -lcusolver
"$NVCC" $ARCH -shared -ccbin g++ -o "$OUT/libshimtest.so" "$OUT/cuda_kernels.o" "$OUT/transformer_b200.o" \
  "$OUT/ref_driver.o" -L"$PKG/lib" -lqib200 -Xlinker -rpath='$ORIGIN/../../qwen-image.cu_b200/lib' -lcublas -lcusolver
echo "built $OUT/libqiref.so $OUT/libshimtest.so"
