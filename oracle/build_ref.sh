#!/bin/bash
# Builds the reference CP-ALS program (zhixianzhu/cpTC) from its own sources,
# unmodified, for sm_100a, into oracle/_ref/cptc_opt.  Test and baseline
# infrastructure only.  The caller names the reference tree in REF_DIR;
# machines without it use the prebuilt binary.
#   - MAGMA is replaced by oracle/refstub/magma_v2.h (only dead code uses it)
#   - oracle/refstub/preinclude.h adds <cstdint> for include/generic.hpp
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
: "${REF_DIR:?set REF_DIR to the reference source tree}"
OUT="$HERE/_ref"
if [ ! -d "$REF_DIR/src" ]; then
  echo "reference sources not found at $REF_DIR" >&2
  exit 2
fi
mkdir -p "$OUT"
SRCS="als.cu cadr.cu common.cu compute_fit.cu dense.cu generic.cu main.cu partition.cu sgd.cu solver.cu sparse.cu tensor.cu"
ARGS=()
for s in $SRCS; do ARGS+=("$REF_DIR/src/$s"); done
nvcc -O3 -gencode arch=compute_100a,code=sm_100a -ccbin g++ \
  -I "$REF_DIR/include" -I "$HERE/refstub" -include "$HERE/refstub/preinclude.h" \
  -o "$OUT/cptc_opt" "${ARGS[@]}" --cudart=static -lcublas -lcusparse -lcusolver
echo "built $OUT/cptc_opt"
