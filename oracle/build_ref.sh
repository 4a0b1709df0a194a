#!/usr/bin/env bash
# Compiles the reference's own CUDA kernels (AICortex kernels.h and the headers
# it includes, the audio front-end ca.cu and the screen front-end's operators
# from cs.cu) for sm_100a into oracle/_ref/, one shared library per
# (d_model, d_state) pair, driven by oracle/ref_harness.cu.
# TEST INFRASTRUCTURE ONLY: the libraries are the golden-vector source for
# tests/golden/make_golden.py and never part of the product.
#
# The Mamba kernels take d_model/d_state from compile-time constants in
# base_constants.h, so the four headers the kernels need are copied to a
# temporary directory outside the repository, the two constants rewritten
# there, and the copy deleted after the build. A stub <windows.h> replaces the
# Windows SDK header that kernels.h includes (kernels.h:14); it declares only
# the BYTE and DWORD types named by ca.cu's capture entry point.
set -euo pipefail
HERE=$(cd "$(dirname "$0")" && pwd)
# the reference checkout: AICORTEX_REFERENCE, default "reference" beside this repository
REF=${AICORTEX_REFERENCE:-$HERE/../../reference}
OUT="$HERE/_ref"
if [ ! -f "$REF/kernels.h" ]; then
  echo "reference sources not found at $REF; skipping oracle/_ref build" >&2
  exit 0
fi
mkdir -p "$OUT"
PAIRS=${AICREF_PAIRS:-"256:32 256:128 256:512"}
for pair in $PAIRS; do
  D=${pair%%:*}; N=${pair##*:}
  lib="$OUT/libaicref_D${D}_N${N}.so"
  if [ -f "$lib" ] && [ "$lib" -nt "$HERE/ref_harness.cu" ] && [ "$lib" -nt "$REF/kernels.h" ] && [ "$lib" -nt "$REF/cs.cu" ] && [ "$lib" -nt "$0" ]; then continue; fi
  tmp=$(mktemp -d /tmp/aicref.XXXXXX)
  cp "$REF/kernels.h" "$REF/uv.h" "$REF/device_constants.h" "$REF/base_constants.h" "$REF/ca.cu" "$tmp/"
  # the screen front-end's two elementwise operators (cs.cu:5-45), cut from
  # cs.cu without its D3D11 interop part, which cannot build here
  awk '/^struct ProcessBgraToRgbOP/{on=1} /^struct InternalCudaVisualState/{on=0} on' "$REF/cs.cu" > "$tmp/cs_ops.h"
  sed -i -E "s/final_channels = [0-9]+/final_channels = ${D}/; s/mamba_d_state = [0-9]+/mamba_d_state = ${N}/" "$tmp/base_constants.h"
  # the two Windows SDK types ca.cu's capture entry point names (ca.cu:76)
  printf 'typedef unsigned char BYTE;\ntypedef unsigned long DWORD;\n' > "$tmp/windows.h"
  nvcc -std=c++17 -O3 --use_fast_math --extended-lambda \
       -gencode arch=compute_100a,code=sm_100a -lineinfo \
       -Xcompiler -fPIC -shared \
       -include "$HERE/ref_shim/prelude.h" -I"$tmp" \
       -o "$lib" "$HERE/ref_harness.cu"
  rm -rf "$tmp"
  echo "built $lib"
done
