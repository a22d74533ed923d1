#!/bin/sh
# Installs the UNMODIFIED reference (hsungo/thesis, pure Python/PyTorch) under baseline/_ref, offline,
# so that bench.py's reference arm can time the reference's own common/model.py + solutions/packed.py
# on the host cores.  baseline/_ref is git-ignored (not product source) but travels with the
# repository snapshot to the GPU host.  The build writes into its source tree, hence the copy.
#   sh baseline/install_reference.sh /path/to/thesis
set -e
SRC=${1:-$THESIS_REFERENCE}
[ -n "$SRC" ] || { echo "usage: $0 /path/to/thesis (or set THESIS_REFERENCE)" >&2; exit 2; }
HERE=$(cd "$(dirname "$0")" && pwd)
TMP=$(mktemp -d)
cp -r "$SRC" "$TMP/thesis"
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --target "$HERE/_ref" "$TMP/thesis"
rm -rf "$TMP"
