#!/usr/bin/env bash
# Builds the reference crate's CUDA kernels, from the sources where they lie, into
# oracle/_ref/libref_moe.so (test infrastructure only: a second oracle for the GPU tests and the
# generator of tests/golden/ fixtures).  Flags follow the reference's build.rs:46-61 with the
# architecture fixed to sm_100a and none of the CUDA_COMPUTE_CAP-driven macros (build.rs:64-80):
# that is the configuration the reference builds on a B200 when CUDA_COMPUTE_CAP is not exported,
# and the only one that compiles for sm_100a (-DSM80_OR_HIGHER fails at qwen3_moe.cu:1094,
# -DSM90_OR_HIGHER at qwen3_moe.cu:2291 and on wgmma).
# Usage: oracle/build_ref.sh [REFERENCE_ROOT]   (default /root/reference)
set -euo pipefail
REF="${1:-/root/reference}"
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
OUT="$HERE/_ref"
if [ ! -d "$REF/kernels" ]; then
  echo "reference sources not found under $REF; skipping" >&2
  exit 0
fi
mkdir -p "$OUT"
FLAGS=(-gencode arch=compute_100a,code=sm_100a -std=c++17 -O3 -Xcompiler -fPIC
       -U__CUDA_NO_HALF_OPERATORS__ -U__CUDA_NO_HALF_CONVERSIONS__
       -U__CUDA_NO_HALF2_OPERATORS__ -U__CUDA_NO_BFLOAT16_CONVERSIONS__
       --expt-relaxed-constexpr --expt-extended-lambda --use_fast_math)
objs=()
for f in topk_softmax moe qwen3_moe nomic_moe; do
  src="$REF/kernels/$f.cu"
  obj="$OUT/$f.o"
  if [ ! -f "$obj" ] || [ "$src" -nt "$obj" ]; then
    nvcc "${FLAGS[@]}" -c "$src" -o "$obj"
  fi
  objs+=("$obj")
done
shim_obj="$OUT/ref_shim.o"
if [ ! -f "$shim_obj" ] || [ "$HERE/ref_shim.cu" -nt "$shim_obj" ]; then
  nvcc "${FLAGS[@]}" -I "$REF/kernels" -c "$HERE/ref_shim.cu" -o "$shim_obj"
fi
objs+=("$shim_obj")
nvcc -gencode arch=compute_100a,code=sm_100a -shared -o "$OUT/libref_moe.so" "${objs[@]}" \
  -Xlinker -Bsymbolic -Xlinker --exclude-libs,ALL
echo "$OUT/libref_moe.so"
