#!/usr/bin/env bash
# Installs the reference package (geniussyn/SWANN, unmodified) into baseline/_ref,
# offline, for bench.py's reference arm and the reference-kernel checker.
#
#   baseline/install.sh [REFERENCE_ROOT]      (default: $SWANN_REFERENCE)
#
# The reference's build writes into its source tree, so it is installed from a
# copy.  Its only dependencies (numpy, torch) are already present and not in the
# offline wheelhouse, hence --no-deps.  baseline/_ref is git-ignored and travels
# to the GPU box with the working tree.
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
src="${1:-${SWANN_REFERENCE:-}}"
if [ -z "$src" ] || [ ! -f "$src/pyproject.toml" ]; then
    echo "usage: $0 REFERENCE_ROOT   (or set SWANN_REFERENCE)" >&2
    exit 2
fi
tmp="$(mktemp -d)"
trap 'rm -rf "$tmp"' EXIT
cp -r "$src" "$tmp/swann_src"
rm -rf "$here/_ref"
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --target "$here/_ref" "$tmp/swann_src"
echo "installed: $here/_ref/swann"
