#!/bin/sh
# Installs the unmodified reference (FAndromedA/sgsa) into baseline/_ref, which is
# git-ignored: it is not part of this repository's source, it only travels with the
# working tree so that bench.py's reference arm and the drop-in test can import it.
#
# The reference has no setup.py or pyproject.toml, so
#   pip install --no-index --no-build-isolation --find-links /opt/wheelhouse \
#       --target baseline/_ref <reference>
# stops with "Directory ... is not installable".  Its Python package is the
# `modelings/` tree, imported as `modelings.*` from the reference root, so the
# install is that tree, unchanged, under baseline/_ref/modelings.
set -e
SRC=${1:-/root/reference}
HERE=$(cd "$(dirname "$0")" && pwd)
[ -d "$SRC/modelings" ] || { echo "reference not found at $SRC" >&2; exit 1; }
rm -rf "$HERE/_ref"
mkdir -p "$HERE/_ref"
cp -r "$SRC/modelings" "$HERE/_ref/modelings"
find "$HERE/_ref" -name '__pycache__' -prune -exec rm -rf {} +
echo "installed $SRC/modelings -> $HERE/_ref/modelings"
