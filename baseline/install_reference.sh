#!/usr/bin/env bash
# Installs the unmodified reference module (snap-research/TDA,
# triton_threshold_attention.py) into baseline/_ref for
# `bench.py --impl reference-triton`.
#
# The reference ships no setup.py / pyproject.toml, so pip refuses the
# directory as it is.  The source is copied to a scratch directory (the
# reference tree is read-only) and given packaging metadata only: a
# pyproject.toml naming the one module.  The module itself is not changed.
# Usage: baseline/install_reference.sh <path of the reference checkout>
# Run where the reference is available; baseline/_ref is git-ignored and
# travels with the repository snapshot to the GPU box.
set -euo pipefail
if [ $# -ne 1 ]; then
  echo "usage: $0 <path of the reference checkout (the directory holding triton_threshold_attention.py)>" >&2
  exit 2
fi
REF=$1
HERE=$(cd "$(dirname "$0")" && pwd)
TMP=$(mktemp -d)
trap 'rm -rf "$TMP"' EXIT
cp "$REF/triton_threshold_attention.py" "$REF/README.md" "$REF/LICENSE" "$TMP/"
cat > "$TMP/pyproject.toml" <<'TOML'
[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "tda-reference"
version = "0.0.0"

[tool.setuptools]
py-modules = ["triton_threshold_attention"]
TOML
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --target "$HERE/_ref" --upgrade "$TMP"
cmp "$REF/triton_threshold_attention.py" "$HERE/_ref/triton_threshold_attention.py"
echo "installed $(ls "$HERE/_ref")"
