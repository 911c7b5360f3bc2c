#!/bin/sh
# Regenerates forge_greedy.c from forge_greedy.hexa with the hexa transpiler
# (hexa-cc, shipped prebuilt in the hexa-lang tree as build/hexat_linux).
# Only needed after editing the .hexa source; the generated C is committed
# so that builds and tests need no hexa toolchain.
#   HEXAT=/path/to/hexat_linux sh make_c.sh
set -e
here=$(cd "$(dirname "$0")" && pwd)
HEXAT=${HEXAT:-/root/reference/build/hexat_linux}
"$HEXAT" "$here/forge_greedy.hexa" "$here/forge_greedy.c"
