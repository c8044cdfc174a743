#!/bin/sh
# Installs the unmodified reference (Yuhang-dev/exp3) into baseline/_ref as the package `exp3`.
#
#   sh baseline/install_reference.sh [path-to-reference]
#
# The reference tree has no packaging metadata (no setup.py / pyproject.toml), so pip cannot
# install it as it stands. Its Python sources are copied unchanged into a scratch directory
# under /tmp, a minimal pyproject.toml naming the package is written beside them, and pip
# installs that offline into baseline/_ref. No source file is edited. baseline/_ref is
# git-ignored; it travels to the GPU box with the working tree, where bench.py's reference_gpu
# record and tests/test_gpu_reference_triton.py import it.
set -eu
src=${1:-/root/reference}
here=$(cd "$(dirname "$0")" && pwd)
tmp=$(mktemp -d /tmp/exp3_ref.XXXXXX)
mkdir -p "$tmp/exp3/upstream"
cp "$src"/*.py "$tmp/exp3/"
cp "$src"/upstream/*.py "$tmp/exp3/upstream/"
cat > "$tmp/pyproject.toml" <<'TOML'
[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "exp3"
version = "0.0.0"

[tool.setuptools]
packages = ["exp3", "exp3.upstream"]
TOML
rm -rf "$here/_ref"
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --target "$here/_ref" "$tmp"
rm -rf "$tmp"
