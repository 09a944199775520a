#!/bin/bash
# Builds the reference comparator from the reference's own sources, in place
# in the reference checkout given by FKC_REFERENCE_ROOT (read-only; nothing is
# copied), into oracle/_ref/:
#   libfkc_ref.so      - flash_kmeans_cuda/csrc/{api.cpp, assign/*.cu, update/*.cu}
#                        compiled with the reference's flags (setup.py:78-85) for
#                        compute_100/sm_100 (setup.py:55), linked against libtorch;
#   fkc_ref_shim*.so   - oracle/ref_shim.cpp, a pybind11 module exposing the fkc::
#                        libtorch API (the reference's nanobind bindings.cpp cannot be
#                        built here: nanobind is not installed).
# Test infrastructure only (see oracle/lloyd.py for the rule on who may use it).
set -euo pipefail
if [ -z "${FKC_REFERENCE_ROOT:-}" ]; then
  echo "FKC_REFERENCE_ROOT is not set: point it at a checkout of the reference to build oracle/_ref" >&2
  exit 2
fi
REF=$FKC_REFERENCE_ROOT
HERE=$(cd "$(dirname "$0")" && pwd)
OUT=$HERE/_ref
CSRC=$REF/flash_kmeans_cuda/csrc
[ -d "$CSRC" ] || { echo "reference sources not found at $CSRC" >&2; exit 2; }
mkdir -p "$OUT/obj"
PY=${PYTHON:-python}
TORCH_INC=$($PY -c 'from torch.utils import cpp_extension as c; print(" ".join("-I"+p for p in c.include_paths()))')
TORCH_LIB=$($PY -c 'import torch, os; print(os.path.join(os.path.dirname(torch.__file__), "lib"))')
ABI=$($PY -c 'import torch; print(int(torch._C._GLIBCXX_USE_CXX11_ABI))')
PYINC=$($PY -c 'import sysconfig; print(sysconfig.get_paths()["include"])')
EXT=$($PY -c 'import sysconfig; print(sysconfig.get_config_var("EXT_SUFFIX"))')
INC="-I$CSRC -I$CSRC/common -I$CSRC/assign -I$CSRC/update $TORCH_INC -I/usr/local/cuda/include"
NVFLAGS="-O3 --use_fast_math -std=c++17 --expt-relaxed-constexpr --expt-extended-lambda -lineinfo \
  -Xcompiler=-fPIC -gencode arch=compute_100,code=sm_100 -D_GLIBCXX_USE_CXX11_ABI=$ABI -DFKC_BUILD_SHARED"
pids=()
for src in assign/assign_safe.cu assign/assign_sm80.cu update/update_sorted.cu update/update_finalize.cu; do
  obj=$OUT/obj/$(basename "${src%.cu}").o
  if [ ! -f "$obj" ] || [ "$CSRC/$src" -nt "$obj" ]; then
    nvcc $NVFLAGS $INC -c "$CSRC/$src" -o "$obj" & pids+=($!)
  fi
done
if [ ! -f "$OUT/obj/api.o" ]; then
  g++ -O3 -std=c++17 -fPIC -D_GLIBCXX_USE_CXX11_ABI=$ABI -DFKC_BUILD_SHARED $INC -c "$CSRC/api.cpp" -o "$OUT/obj/api.o" & pids+=($!)
fi
for p in "${pids[@]}"; do wait "$p"; done
g++ -shared -o "$OUT/libfkc_ref.so" "$OUT"/obj/*.o -L"$TORCH_LIB" -lc10 -ltorch_cpu -ltorch_cuda -lc10_cuda \
  -L/usr/local/cuda/lib64 -lcudart -Wl,-rpath,"$TORCH_LIB"
g++ -O2 -std=c++17 -shared -fPIC -D_GLIBCXX_USE_CXX11_ABI=$ABI -DTORCH_EXTENSION_NAME=fkc_ref_shim \
  $INC -I"$PYINC" "$HERE/ref_shim.cpp" -o "$OUT/fkc_ref_shim$EXT" \
  -L"$OUT" -lfkc_ref -L"$TORCH_LIB" -lc10 -ltorch_cpu -ltorch_python -ltorch_cuda -lc10_cuda \
  -Wl,-rpath,'$ORIGIN' -Wl,-rpath,"$TORCH_LIB"
echo "built $OUT/libfkc_ref.so and $OUT/fkc_ref_shim$EXT"
