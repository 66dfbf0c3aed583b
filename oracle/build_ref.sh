#!/usr/bin/env bash
# Build the UNMODIFIED reference extension (doublewordai/tans-vectoradd,
# csrc/{fp8_memcpy.cu,tans_codec.cpp,tans_decode.cu,vecadd.cu}) straight from
# its sources into oracle/_ref/, for sm_100a, with nvcc/g++ invoked directly
# (the reference's own setup.py is not run).
#
# Test infrastructure only: the resulting oracle/_ref/_C*.so is the
# reference's pybind module `_C` (ops tans_encode_interleaved, gpu_tans_decode,
# fp8_memcpy, fp8_vecadd_raw, fp8_vecadd_fused_tans; csrc/fp8_memcpy.cu:66-78).
# Tests and the CPU-baseline leg of bench.py load it as the checker.  Nothing
# in the product links it.
#
# Usage: oracle/build_ref.sh [REFERENCE_ROOT]   (default: $TANS_REFERENCE_ROOT, else a
# sibling checkout named "reference" next to this repository)
# Flags follow the reference's setup.py:40-63 (-O3 --use_fast_math -lineinfo,
# cxx -O3 -fopenmp) with the arch fixed to sm_100a.
set -euo pipefail

HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
REF="${1:-${TANS_REFERENCE_ROOT:-$HERE/../../reference}}"
OUT="$HERE/_ref"
BUILD="$OUT/build"

if [[ ! -f "$REF/csrc/vecadd.cu" ]]; then
    echo "build_ref: reference sources not found under $REF" >&2
    exit 2
fi

PY="${PYTHON:-python}"
TORCH_INC=$("$PY" -c 'import torch.utils.cpp_extension as c; print(" ".join("-I"+p for p in c.include_paths()))' 2>/dev/null)
TORCH_LIB=$("$PY" -c 'import torch, os; print(os.path.join(os.path.dirname(torch.__file__), "lib"))')
PY_INC=$("$PY" -c 'import sysconfig; print(sysconfig.get_paths()["include"])')
EXT_SUFFIX=$("$PY" -c 'import sysconfig; print(sysconfig.get_config_var("EXT_SUFFIX"))')
CUDA_HOME="${CUDA_HOME:-/usr/local/cuda}"
NVCC="$CUDA_HOME/bin/nvcc"

DEFS="-DTORCH_EXTENSION_NAME=_C -DTORCH_API_INCLUDE_EXTENSION_H -D_GLIBCXX_USE_CXX11_ABI=1"
INCS="$TORCH_INC -I$PY_INC -I$CUDA_HOME/include"

mkdir -p "$BUILD"
echo "build_ref: compiling reference sources from $REF/csrc -> $OUT"

pids=()
for f in fp8_memcpy tans_decode vecadd; do
    "$NVCC" -c "$REF/csrc/$f.cu" -o "$BUILD/$f.o" $DEFS $INCS \
        -Xcompiler -fPIC -std=c++17 -O3 --use_fast_math -lineinfo \
        -gencode arch=compute_100a,code=sm_100a \
        -D__CUDA_NO_HALF_OPERATORS__ -D__CUDA_NO_HALF_CONVERSIONS__ \
        -D__CUDA_NO_BFLOAT16_CONVERSIONS__ -D__CUDA_NO_HALF2_OPERATORS__ \
        --expt-relaxed-constexpr &
    pids+=($!)
done
g++ -c "$REF/csrc/tans_codec.cpp" -o "$BUILD/tans_codec.o" $DEFS $INCS \
    -fPIC -std=c++17 -O3 -fopenmp &
pids+=($!)
for p in "${pids[@]}"; do wait "$p"; done

g++ -shared -o "$OUT/_C$EXT_SUFFIX" \
    "$BUILD/fp8_memcpy.o" "$BUILD/tans_decode.o" "$BUILD/vecadd.o" "$BUILD/tans_codec.o" \
    -L"$TORCH_LIB" -Wl,-rpath,"$TORCH_LIB" \
    -L"$CUDA_HOME/lib64" \
    -lc10 -lc10_cuda -ltorch -ltorch_cpu -ltorch_cuda -ltorch_python -lcudart -fopenmp
rm -rf "$BUILD"
echo "build_ref: wrote $OUT/_C$EXT_SUFFIX"
