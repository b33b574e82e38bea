#!/usr/bin/env bash
# Test infrastructure, not product code.
#
# Builds the reference's own cuda-cpp backend (yaneurao/BulletOu,
# crates/cuda_cpp/cpp/bulletou_cuda_backend.cu + its two headers) into a
# shared library under oracle/_ref/, straight from the reference sources where
# they lie.  Nothing from the reference is copied into this repository.
#
# Flags follow crates/cuda_cpp/build.rs:41-50 (-std=c++17 -O3 --use_fast_math,
# cudart + cublas); the additions are the sm_100a target, -shared/-fPIC, and a
# generated trampoline unit (gen_ref_exports.py) that re-exports each C-ABI
# entry as refx_<name>, because the reference's entries get internal linkage
# outside MSVC.  The result is used by
# tests/ (GPU parity against the reference kernels) and by
# `bench.py --impl reference` (the reference backend timed on the same GPU).
#
# Usage: oracle/build_ref.sh REFERENCE_ROOT   (or BULLETOU_REFERENCE_ROOT set)
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
ref_root="${1:-${BULLETOU_REFERENCE_ROOT:-}}"
if [[ -z "$ref_root" ]]; then
    echo "usage: oracle/build_ref.sh REFERENCE_ROOT (or set BULLETOU_REFERENCE_ROOT)" >&2
    exit 2
fi
src="$ref_root/crates/cuda_cpp/cpp/bulletou_cuda_backend.cu"
out_dir="$here/_ref"
out="$out_dir/libref_cudacpp.so"
if [[ ! -f "$src" ]]; then
    echo "reference source not found: $src" >&2
    exit 2
fi
mkdir -p "$out_dir"
if [[ -f "$out" && "$out" -nt "$src" && "$out" -nt "$here/../include/bulletou_cuda_cpp.h" ]]; then
    echo "up to date: $out"
    exit 0
fi
nvcc=${NVCC:-nvcc}
python3 "$here/gen_ref_exports.py" "$here/../include/bulletou_cuda_cpp.h" "$src" "$out_dir/ref_exports.cu"
"$nvcc" -std=c++17 -O3 --use_fast_math \
    -gencode arch=compute_100a,code=sm_100a \
    -Xcompiler -fPIC -shared -w \
    -I"$ref_root/crates/cuda_cpp/cpp" \
    -o "$out.tmp" "$out_dir/ref_exports.cu" \
    -lcublas -lcudart
mv "$out.tmp" "$out"
echo "built $out"
