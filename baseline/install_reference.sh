#!/usr/bin/env bash
# Offline install of the reference into baseline/_ref (its pyproject declares
# dependencies that are not in the wheelhouse, so --no-deps), plus an unmodified
# copy of its recipes/ tree, which the wheel does not package.
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
if [ $# -lt 1 ]; then
    echo "usage: $0 <path to the reference source tree>" >&2
    exit 2
fi
SRC="$1"
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --target "$HERE/_ref" "$SRC"
# package data the wheel does not declare (the launcher and engine read it at run time)
cp "$SRC/mvp_engine/config/default.yaml" "$HERE/_ref/mvp_engine/config/default.yaml"
rm -rf "$HERE/_ref/recipes"
cp -r "$SRC/recipes" "$HERE/_ref/recipes"
echo "reference installed under $HERE/_ref"
