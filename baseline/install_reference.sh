#!/bin/sh
# Install the unmodified reference (apaz-cli/ZOTitan) into baseline/_ref, offline, for
# baseline/reference_steps.py. The reference's checkout is read-only, so it is installed
# from a copy; its declared dependencies (torch, transformers, liger-kernel, tyro, ...)
# are the image's own, so dependency resolution is skipped (--no-deps).
#   sh baseline/install_reference.sh /path/to/reference
set -e
SRC="$1"
[ -n "$SRC" ] || { echo "usage: sh baseline/install_reference.sh /path/to/reference" >&2; exit 2; }
HERE="$(cd "$(dirname "$0")" && pwd)"
TMP="$(mktemp -d)"
cp -r "$SRC"/. "$TMP"/
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --target "$HERE/_ref" --upgrade "$TMP"
rm -rf "$TMP"
