#!/usr/bin/env bash
# Builds the reference's own C++ engine (CPU mode) from its sources, in place
# under the reference tree, into oracle/_ref/ (git-ignored). Test
# infrastructure only: the tests use it to pin the C restatement, and the
# CPU-baseline leg of bench.py may time it.
#
# Inputs read from the reference tree (nothing is copied into this repo):
#   python/bindings.cpp src/engine.cpp src/arena.cpp src/safetensors.cpp src/sha256.cpp
#   src/kernels/{feature_map,attention_forward,attention_backward}.cpp, include/
# The reference's own build system (CMake + FetchContent) is not used; with no
# USE_CUDA/USE_HIP define its HAL header selects the host fallback.
set -euo pipefail
# The reference tree is named by SUBQ_REFERENCE_ROOT (required).
REF=${SUBQ_REFERENCE_ROOT:-}
HERE=$(cd "$(dirname "$0")" && pwd)
OUT="$HERE/_ref"
if [ -z "$REF" ]; then
  echo "SUBQ_REFERENCE_ROOT is not set: point it at the reference tree to build oracle/_ref" >&2
  exit 0
fi
if [ ! -d "$REF/src/kernels" ]; then
  echo "reference tree not found at $REF; oracle/_ref not rebuilt" >&2
  exit 0
fi
mkdir -p "$OUT"
PY=${PYTHON:-python3}
SITE=$($PY -c 'import site; print(site.getsitepackages()[0])')
JSON_INC="$SITE/include/cudnn_frontend/thirdparty"
EXT=$($PY -c 'import sysconfig; print(sysconfig.get_config_var("EXT_SUFFIX"))')
PYBIND_INC=$($PY -c 'import pybind11; print(pybind11.get_include())')
PY_INC=$($PY -c 'import sysconfig; print(sysconfig.get_paths()["include"])')
TARGET="$OUT/_C$EXT"
SRCS=(python/bindings.cpp src/engine.cpp src/arena.cpp src/safetensors.cpp src/sha256.cpp
      src/kernels/feature_map.cpp src/kernels/attention_forward.cpp src/kernels/attention_backward.cpp)
ABS=()
for s in "${SRCS[@]}"; do ABS+=("$REF/$s"); done
# Rebuild only when a source is newer than the library.
if [ -f "$TARGET" ]; then
  stale=0
  for s in "${ABS[@]}"; do [ "$s" -nt "$TARGET" ] && stale=1; done
  [ $stale -eq 0 ] && { echo "$TARGET"; exit 0; }
fi
${CXX:-g++} -O3 -std=c++20 -shared -fPIC -ffast-math \
  -I"$REF/include" -I"$JSON_INC" -I"$PYBIND_INC" -I"$PY_INC" \
  "${ABS[@]}" -o "$TARGET"
echo "$TARGET"
