#!/bin/sh
# Installs the reference's own Python layer (package `pdefa`, unmodified) and its
# pytest suite into baseline/_ref (git-ignored; it travels with the working tree to
# the GPU machine), for tests/test_gpu_reference_python.py. The reference's native
# libraries are never used: the test puts this repository's libpdefa_native.so in
# their place.
#
# Usage: PDEFA_REFERENCE=<pdefa checkout> sh tests/install_reference_python.sh
set -e
: "${PDEFA_REFERENCE:?set PDEFA_REFERENCE to the pdefa reference checkout}"
ROOT=$(cd "$(dirname "$0")/.." && pwd)
TMP=$(mktemp -d)
# the setuptools build writes into its source tree, so it runs on a copy
cp -r "$PDEFA_REFERENCE" "$TMP/src"
python -m pip install --no-index --no-build-isolation --no-deps --upgrade --target "$ROOT/baseline/_ref" "$TMP/src"
rm -rf "$ROOT/baseline/_ref/pdefa_tests"
cp -r "$PDEFA_REFERENCE/pdefa/tests" "$ROOT/baseline/_ref/pdefa_tests"
rm -rf "$TMP"
echo "installed: $ROOT/baseline/_ref/pdefa and $ROOT/baseline/_ref/pdefa_tests"
