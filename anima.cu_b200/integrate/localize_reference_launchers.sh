#!/bin/sh
# Makes the reference's own definitions of the launchers libanima_b200.so serves local
# (invisible to the linker) in a static archive or object of the reference build, e.g.
#   localize_reference_launchers.sh build/libanima_kernels.a
# Afterwards transformer.cpp, qwen3.cpp, llm_adapter.cpp and vae.cpp, linked against that
# archive plus libanima_b200.so, call the B200 kernels; every other launcher of the
# archive (softmax, patchify, conv, sampler steps, ...) stays the reference's own.
# Usage: localize_reference_launchers.sh <archive-or-object> [output]
set -e
HERE=$(cd "$(dirname "$0")" && pwd)
IN=$1
OUT=${2:-$1}
[ -n "$IN" ] || { echo "usage: $0 <archive-or-object> [output]" >&2; exit 2; }
ARGS=""
for sym in $(grep -v '^#' "$HERE/replaced_launchers.txt"); do ARGS="$ARGS --localize-symbol=$sym"; done
# shellcheck disable=SC2086
objcopy $ARGS "$IN" "$OUT"
