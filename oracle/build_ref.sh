#!/usr/bin/env bash
# Compile the reference's own CUDA kernels (admm_fused.cu, pcg_blktridi.cu,
# common/block_tridi.cu) from the read-only reference tree, unmodified, for
# sm_100a, together with oracle/ref_shim.cu, into oracle/_ref/libtmpc_refcuda.so.
# Test infrastructure only (golden vectors, GPU cross-check).  Outputs go to
# oracle/_ref/ (git-ignored) only.
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
REF="${TMPC_REFERENCE_ROOT:-$(dirname "$HERE")/../reference}/turbompc/solvers"
OUT="$HERE/_ref"
if [ ! -d "$REF" ]; then echo "reference tree not found at $REF; skipping"; exit 0; fi
mkdir -p "$OUT"
SRC=("$REF/admm/csrc/admm_fused.cu" "$REF/linear_systems_solvers/csrc/pcg_blktridi.cu" "$REF/csrc/common/block_tridi.cu" "$HERE/ref_shim.cu")
if [ -f "$OUT/libtmpc_refcuda.so" ]; then
  newest=$(ls -t "${SRC[@]}" "$OUT/libtmpc_refcuda.so" | head -1)
  if [ "$newest" = "$OUT/libtmpc_refcuda.so" ]; then echo "$OUT/libtmpc_refcuda.so up to date"; exit 0; fi
fi
nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -rdc=true -Xcompiler -fPIC -shared \
  -I"$REF/admm/csrc" -I"$REF/linear_systems_solvers/csrc" -I"$REF/csrc/common" \
  "${SRC[@]}" -o "$OUT/libtmpc_refcuda.so"
echo "$OUT/libtmpc_refcuda.so"
