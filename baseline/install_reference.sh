#!/usr/bin/env bash
# Installs the unmodified reference package (sr_states) into baseline/_ref for the
# reference arm of bench.py (`--impl reference`) and the CPU baseline, offline.
# The reference's build writes into its source tree, so it is installed from a
# scratch copy.  Usage: baseline/install_reference.sh <reference checkout>
set -euo pipefail
src=${1:?usage: install_reference.sh <reference checkout>}
here=$(cd "$(dirname "$0")" && pwd)
scratch=$(mktemp -d)
trap 'rm -rf "$scratch"' EXIT
cp -r "$src" "$scratch/reference"
rm -rf "$here/_ref"
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
  --target "$here/_ref" "$scratch/reference"
python -c "import sys; sys.path.insert(0, '$here/_ref'); import sr_states; print('installed', sr_states.__file__)"
