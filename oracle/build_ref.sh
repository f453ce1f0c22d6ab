#!/bin/sh
# Compile the reference's own scalar C program (c/intref.c) from its source where it lies in the
# reference checkout, into oracle/_ref/intref.  TEST INFRASTRUCTURE: the binary is the reference
# implementation used as a parity cross-check and as bench.py's CPU baseline; nothing in the
# shipped engine links or runs it.  Flags follow the reference's c/Makefile (-O2 -Wall -Wextra).
#   sh oracle/build_ref.sh [REFERENCE_DIR]
# (default: $EII_REFERENCE, else a directory named `reference` beside this repository)
set -eu
HERE="$(cd "$(dirname "$0")" && pwd)"
REF="${1:-${EII_REFERENCE:-$HERE/../../reference}}"
SRC="$REF/c/intref.c"
if [ ! -f "$SRC" ]; then
    echo "build_ref: $SRC not found; oracle/_ref/intref not rebuilt" >&2
    exit 0
fi
mkdir -p "$HERE/_ref"
${CC:-gcc} -O2 -Wall -Wextra -o "$HERE/_ref/intref" "$SRC"
echo "built $HERE/_ref/intref from $SRC"
