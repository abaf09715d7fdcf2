#!/usr/bin/env bash
# Builds the CPU oracles -- TEST INFRASTRUCTURE ONLY.
#   oracle/_build/libtilemix_oracle.so : the C restatement (tilemix_oracle.c)
#   oracle/_ref/libtilemix_ref.so      : the reference's OWN CPU oracle headers
#                                        (src/tests/reference_*.h), compiled where
#                                        they lie, behind ref_shim.cpp
#   oracle/_ref/libtilemix_ref_gpu.so  : the reference's OWN GPU kernels
#                                        (src/tilemix.cu) for sm_100a, compiled
#                                        where they lie, behind ref_gpu_shim.cu
#                                        (bench.py's "reference GPU" column)
#   oracle/_ref/tilemix_ref_demo       : the reference's OWN driver src/main.cu
#                                        (with src/tilemix.cu), for comparing
#                                        its printed output[0] with tilemix_demo
# Usage: oracle/build_ref.sh [REFERENCE_ROOT]   (default: $TILEMIX_REFERENCE_ROOT;
# oracle/__init__.py passes the reference_path of BASELINE.json when unset)
# The reference build is skipped, not failed, when the reference tree is absent.
set -euo pipefail
here="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
ref_root="${1:-${TILEMIX_REFERENCE_ROOT:-}}"
cuda_inc="${CUDA_HOME:-/usr/local/cuda}/include"

mkdir -p "$here/_build"
gcc -std=c11 -O3 -march=x86-64-v3 -ffp-contract=off -fopenmp -fPIC -shared -Wall -Wextra \
    "$here/tilemix_oracle.c" -o "$here/_build/libtilemix_oracle.so" -lm

if [[ -n "$ref_root" && -f "$ref_root/src/tests/reference_tilemix.h" ]]; then
    mkdir -p "$here/_ref"
    g++ -std=c++17 -O3 -march=x86-64-v3 -ffp-contract=off -fopenmp -fPIC -shared \
        -I"$cuda_inc" -I"$ref_root/src/tests" -I"$ref_root/include" \
        "$here/ref_shim.cpp" -o "$here/_ref/libtilemix_ref.so"
    echo "built $here/_ref/libtilemix_ref.so from $ref_root/src/tests"
    if [[ -f "$ref_root/src/tilemix.cu" ]] && command -v nvcc > /dev/null; then
        nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -Xcompiler -fPIC -shared \
            -I"$ref_root/include" "$ref_root/src/tilemix.cu" "$here/ref_gpu_shim.cu" \
            -o "$here/_ref/libtilemix_ref_gpu.so"
        echo "built $here/_ref/libtilemix_ref_gpu.so from $ref_root/src/tilemix.cu"
        # the reference's own driver (src/main.cu), unmodified, for the
        # output[0] comparison with tilemix_demo
        nvcc -gencode arch=compute_100a,code=sm_100a -O2 -std=c++17 -I"$ref_root/include" \
            "$ref_root/src/main.cu" "$ref_root/src/tilemix.cu" -o "$here/_ref/tilemix_ref_demo"
        echo "built $here/_ref/tilemix_ref_demo from $ref_root/src/main.cu"
    fi
else
    echo "reference tree not found at $ref_root; oracle/_ref not rebuilt"
fi
echo "built $here/_build/libtilemix_oracle.so"
