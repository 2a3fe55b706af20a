#!/bin/sh
# Installs the reference package (MaskAhead's src/maskahead) into baseline/_ref, where the
# drop-in tests import it from (tests/reference_pkg.py). Offline: no index, no
# dependencies (torch, triton and yaml are already in the environment), and the build
# runs on a copy, so the checkout itself is never written to.
#
#   sh baseline/install_reference.sh <reference checkout>
set -eu
src=${1:?usage: sh baseline/install_reference.sh <reference checkout>}
here=$(cd "$(dirname "$0")" && pwd)
tmp=$(mktemp -d)
trap 'rm -rf "$tmp"' EXIT
cp -r "$src" "$tmp/ref"
python -m pip install --no-index --no-build-isolation --no-deps --upgrade --target "$here/_ref" "$tmp/ref"
python -c "import sys; sys.path.insert(0, '$here/_ref'); import maskahead.runtime.session as s; print('installed', s.__file__)"
