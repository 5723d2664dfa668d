#!/usr/bin/env bash
# Builds the reference's own SGEMM / HGEMM / flash-attention kernels for sm_100a
# straight from its unmodified sources (the checkout named by REF; nothing is
# copied into this repository) plus oracle/ref_shim.cpp, into
# oracle/_ref/libsion_ref.so. TEST INFRASTRUCTURE ONLY (comparator in tests and
# bench.py). The reference's CuTe kernels need CUTLASS/CuTe headers; its own
# third_party/cutlass submodule is empty, so the copy bundled with the image's
# flashinfer package is used (CUTLASS_INC overrides).
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
REF="${REF:?set REF to the reference checkout (the directory holding src/felix)}"
OUT="$HERE/_ref"
CUTLASS_INC="${CUTLASS_INC:-$(python -c 'import os, flashinfer; print(os.path.join(os.path.dirname(flashinfer.__file__), "data", "cutlass", "include"))' 2>/dev/null || true)}"
NVCC="${CUDA_HOME:-/usr/local/cuda}/bin/nvcc"
[ -d "$REF/src/felix" ] || { echo "reference sources not found at $REF" >&2; exit 1; }
[ -d "$CUTLASS_INC/cute" ] || { echo "CuTe headers not found (CUTLASS_INC=$CUTLASS_INC)" >&2; exit 1; }
if [ -f "$OUT/libsion_ref.so" ] && [ -z "${FORCE:-}" ] && [ "$OUT/libsion_ref.so" -nt "$HERE/ref_shim.cpp" ]; then
  echo "$OUT/libsion_ref.so (up to date)"
  exit 0
fi
mkdir -p "$OUT/obj"
FLAGS=(-std=c++20 -O3 -lineinfo -use_fast_math -gencode arch=compute_100a,code=sm_100a
       -Xcompiler -fPIC -I"$REF/include" -I"$REF/src/felix" -I"$CUTLASS_INC")
SRCS=(
  "$REF/src/felix/base/felix_api.cpp"
  "$REF/src/felix/base/registry.cpp"
  "$REF/src/felix/base/status.cpp"
  "$REF/src/felix/gemm/sgemm/cute_sgemm_64x64_nn_kernel_launch.cu"
  "$REF/src/felix/gemm/hgemm/cute_hgemm_128x128_nn_kernel_launch.cu"
  "$REF/src/felix/gemm/hgemm/cute_hgemm_128x128_nt_kernel_launch.cu"
  "$REF/src/felix/flash_attention/ampere_flash_attn_mma16168_64_1D_warp_tiling_kernel_launch.cu"
  "$HERE/ref_shim.cpp"
)
OBJS=()
pids=()
for s in "${SRCS[@]}"; do
  o="$OUT/obj/$(basename "$s").o"
  OBJS+=("$o")
  if [[ "$s" == *.cpp ]]; then
    "$NVCC" -x cu "${FLAGS[@]}" -c "$s" -o "$o" &
  else
    "$NVCC" "${FLAGS[@]}" -c "$s" -o "$o" &
  fi
  pids+=($!)
done
for p in "${pids[@]}"; do wait "$p"; done
"$NVCC" -shared -gencode arch=compute_100a,code=sm_100a -cudart static \
  -Xlinker -Bsymbolic -o "$OUT/libsion_ref.so" "${OBJS[@]}"
rm -rf "$OUT/obj"
echo "$OUT/libsion_ref.so"
