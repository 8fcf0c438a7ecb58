#!/usr/bin/env bash
# Builds the CPU oracle (test infrastructure only) into oracle/_build/.
# -ffp-contract=off keeps every a*b+c as two roundings unless fmaf() is
# written out, which the sampler specification relies on.
set -euo pipefail
here="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
mkdir -p "$here/_build"
gcc -O2 -std=c11 -fPIC -shared -ffp-contract=off -fno-fast-math \
    -o "$here/_build/libfg_oracle.so" "$here/fg_oracle.c" -lm
