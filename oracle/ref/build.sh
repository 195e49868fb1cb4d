#!/usr/bin/env bash
# Compiles the reference's own sources (the-database/animejanai-inference, read-only at $1) into
# oracle/_ref/: the checkers and the CPU baseline. Nothing here is part of the product, and no
# reference source is copied: each library is built from the files where they lie, plus the thin
# C shims in this directory. Only the compilers run (no reference build system).
# The reference tree: the first argument, else $AJIB_REFERENCE, else a `reference` directory beside
# this repository.
set -euo pipefail
HERE=$(cd "$(dirname "$0")" && pwd)
REF=${1:-${AJIB_REFERENCE:-$HERE/../../../reference}}
OUT=$HERE/../_ref
mkdir -p "$OUT"
CXX=${CXX:-g++}
NVCC=${NVCC:-nvcc}
ARCH="-gencode arch=compute_100a,code=sm_100a"

# CPU reference net (sanity/native_ref.h + src/native/pack.cpp)
$CXX -O3 -std=c++17 -fPIC -shared -I"$REF/src" -I"$REF/sanity" -I"$REF/include" \
    -I"$HERE" "$HERE/refnet_shim.cpp" "$REF/src/native/pack.cpp" -o "$OUT/libref_net.so" -lpthread
# CPU tiler (src/core/tiling.cpp)
$CXX -O2 -std=c++17 -fPIC -shared -I"$REF/src" -I"$REF/src/core" -I"$REF/include" \
    "$HERE/reftiling_shim.cpp" "$REF/src/core/tiling.cpp" -o "$OUT/libref_tiling.so" -lpthread
# ONNX lowering (src/native/onnx_graph.cpp + lower.cpp + pack.cpp)
$CXX -O2 -std=c++17 -fPIC -shared -I"$REF/src" -I"$REF/include" \
    "$HERE/reflower_shim.cpp" "$REF/src/native/onnx_graph.cpp" "$REF/src/native/lower.cpp" "$REF/src/native/pack.cpp" \
    -o "$OUT/libref_lower.so"
# host resampling tables and colour constants (src/resample.h)
$CXX -O2 -std=c++17 -fPIC -shared -I"$REF/src" -I"$REF/include" \
    "$HERE/refresample_shim.cpp" -o "$OUT/libref_resample.so"
# GPU: the reference colour kernels (src/kernels.cu), GPU tiler (src/core/tiling_gpu.cu) and conv
# kernels (src/native/conv.cu + pack.cpp) for sm_100a — bit-exact checkers and the GPU bar
if command -v "$NVCC" >/dev/null; then
    $NVCC $ARCH -O3 -std=c++17 -Xcompiler -fPIC -shared -I"$REF/src" -I"$REF/include" \
        "$REF/src/kernels.cu" -o "$OUT/libref_kernels.so"
    $NVCC $ARCH -O3 -std=c++17 -Xcompiler -fPIC -shared -I"$REF/src" -I"$REF/src/core" -I"$REF/include" \
        "$HERE/reftiling_gpu_shim.cu" "$REF/src/core/tiling_gpu.cu" -o "$OUT/libref_tiling_gpu.so"
    $NVCC $ARCH -O3 -std=c++17 -Xcompiler -fPIC -shared -I"$REF/src" -I"$REF/include" \
        "$HERE/refconv_shim.cu" "$REF/src/native/conv.cu" "$REF/src/native/pack.cpp" -o "$OUT/libref_conv.so"
    # the reference's GPU executor over those kernels (src/native/executor.cpp + layout.cpp)
    $NVCC $ARCH -O3 -std=c++17 -Xcompiler -fPIC -shared -I"$REF/src" -I"$REF/include" -I"$HERE" \
        "$HERE/refexec_shim.cu" "$REF/src/native/executor.cpp" "$REF/src/native/layout.cpp" \
        "$REF/src/native/conv.cu" "$REF/src/native/pack.cpp" -o "$OUT/libref_exec.so"
fi
echo "oracle/_ref built from $REF"
