#!/usr/bin/env bash
# Builds the REFERENCE engine (HuanLinOTO/CUDA-MSST-Infer) from its own sources,
# where they lie, into oracle/_ref/libcudasep_ref.so for sm_100a, together with
# the test-only harness oracle/ref/harness.cu.  No reference source is copied.
#
# Recipe (the reference's CMakeLists.txt:19 flags, arch forced to sm_100a):
#   every src/*.cu, plus audio_io.cpp and inference_app.cpp; main.cpp,
#   python_bindings.cpp and http_server.cpp are left out (the last one does not
#   build as shipped: it needs a generated webui header with symbols that
#   tools/embed_html.py never emits).  Links cuBLAS, cuBLASLt, cuFFT, cuDNN.
#
# Usage: oracle/build_ref.sh [REF_SRC_DIR]   (default: $REF_SRC, else the reference
# checkout's src/ directory of this build container)
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
SRC="${1:-${REF_SRC:-/root/reference/src}}"
OUT="$HERE/_ref"
OBJ="$OUT/obj"
mkdir -p "$OBJ"
if [ ! -d "$SRC" ]; then
  echo "reference sources not found at $SRC" >&2
  exit 1
fi
NVCC="${NVCC:-nvcc}"
CUDNN_INC="${CUDNN_INC:-/usr/include/x86_64-linux-gnu}"
FLAGS=(-O3 --use_fast_math --expt-relaxed-constexpr -std=c++17 -Xcompiler -fPIC
       -gencode arch=compute_100a,code=sm_100a -I"$SRC" -I"$CUDNN_INC" -DNDEBUG -w)

srcs=()
for f in "$SRC"/*.cu "$SRC"/audio_io.cpp "$SRC"/inference_app.cpp; do
  srcs+=("$f")
done
srcs+=("$HERE/ref/harness.cu")

pids=()
objs=()
for f in "${srcs[@]}"; do
  base="$(basename "$f")"
  o="$OBJ/${base}.o"
  objs+=("$o")
  if [ "$o" -nt "$f" ] && [ "$o" -nt "$0" ]; then continue; fi
  if [[ "$f" == *.cpp ]]; then
    "$NVCC" "${FLAGS[@]}" -x cu -c "$f" -o "$o" &
  else
    "$NVCC" "${FLAGS[@]}" -c "$f" -o "$o" &
  fi
  pids+=($!)
  # keep at most 8 compilers in flight
  if [ "${#pids[@]}" -ge 8 ]; then wait "${pids[0]}"; pids=("${pids[@]:1}"); fi
done
for p in "${pids[@]}"; do wait "$p"; done

"$NVCC" -shared -gencode arch=compute_100a,code=sm_100a -o "$OUT/libcudasep_ref.so" "${objs[@]}" \
  -lcublas -lcublasLt -lcufft -L/usr/lib/x86_64-linux-gnu -lcudnn
echo "built $OUT/libcudasep_ref.so"
