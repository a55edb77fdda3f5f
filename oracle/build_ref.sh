#!/usr/bin/env bash
# Builds the reference's own Flat-search extension (rapidadb._C) and its two
# k-means kernels from the unmodified reference sources, for sm_100a, into
# oracle/_ref/.  Test infrastructure: the outputs generate and check golden
# vectors on a GPU host (tests/golden/make_golden.py).  Nothing is copied into
# the repository; the sources are compiled where they lie.
#
# The reference's own setup.py / CMakeLists.txt cannot be used as shipped
# (each lists a .cu file that does not exist), so this recipe compiles the
# existing translation units directly:
#   CUDA : csrc/kernels/{distance,topk,topk_warp}.cu      (setup.py:11-16 flags)
#   C++  : csrc/index/flat_index.cpp csrc/core/stream_pool.cpp
#          csrc/bindings/torch_extension.cpp
#   k-means: csrc/kernels/kmeans.cu (no host launcher in the reference) is
#          compiled with relocatable device code and linked with
#          oracle/ref_kmeans_launch.cu, which only launches the two kernels.
# csrc/clustering/kmeans.cpp is excluded: its line 20 is not C++.
set -euo pipefail
REF_SRC=${REF_SRC:?set REF_SRC to the reference source tree (oracle/Makefile sets it)}
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
OUT="$HERE/_ref"
B="$OUT/build"
mkdir -p "$B" "$OUT/rapidadb_ref"

PY=${PYTHON:-python}
TORCH_INC=$($PY -c "import torch.utils.cpp_extension as c; print(' '.join('-I'+p for p in c.include_paths('cuda')))" 2>/dev/null)
TORCH_LIB=$($PY -c "import torch.utils.cpp_extension as c; print(c.library_paths('cuda')[0])" 2>/dev/null)
PY_INC=$($PY -c "import sysconfig; print(sysconfig.get_paths()['include'])")
INC="-I$REF_SRC/csrc/include $TORCH_INC -I$PY_INC"
DEFS="-DTORCH_EXTENSION_NAME=_C -DTORCH_API_INCLUDE_EXTENSION_H -D_GLIBCXX_USE_CXX11_ABI=1"
NVFLAGS="-gencode arch=compute_100a,code=sm_100a -O3 --use_fast_math --expt-relaxed-constexpr --extended-lambda -std=c++17 -Xcompiler -fPIC"

pids=()
for f in distance topk topk_warp; do
  nvcc $NVFLAGS $INC $DEFS -c "$REF_SRC/csrc/kernels/$f.cu" -o "$B/$f.o" & pids+=($!)
done
for f in index/flat_index core/stream_pool bindings/torch_extension; do
  g++ -O2 -std=c++17 -fPIC $INC $DEFS -c "$REF_SRC/csrc/$f.cpp" -o "$B/$(basename $f).o" & pids+=($!)
done
# k-means kernels + launcher (relocatable device code, device-linked)
nvcc $NVFLAGS -rdc=true $INC -c "$REF_SRC/csrc/kernels/kmeans.cu" -o "$B/kmeans.o" & pids+=($!)
nvcc $NVFLAGS -rdc=true -c "$HERE/ref_kmeans_launch.cu" -o "$B/ref_kmeans_launch.o" & pids+=($!)
for p in "${pids[@]}"; do wait "$p"; done

g++ -shared -o "$OUT/rapidadb_ref/_C.so" "$B/distance.o" "$B/topk.o" "$B/topk_warp.o" \
    "$B/flat_index.o" "$B/stream_pool.o" "$B/torch_extension.o" \
    -L"$TORCH_LIB" -lc10 -lc10_cuda -ltorch -ltorch_cpu -ltorch_cuda -ltorch_python \
    -L/usr/local/cuda/lib64 -lcudart -Wl,-rpath,"$TORCH_LIB"
nvcc -gencode arch=compute_100a,code=sm_100a -shared -Xcompiler -fPIC -cudart static \
    "$B/kmeans.o" "$B/ref_kmeans_launch.o" -o "$OUT/libref_kmeans.so"
touch "$OUT/rapidadb_ref/__init__.py"
rm -rf "$B"
echo "built $OUT/rapidadb_ref/_C.so $OUT/libref_kmeans.so"
