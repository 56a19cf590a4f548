#!/bin/sh
# Installs the reference implementation (Hevensh/INTP_Preliminary, pure Python)
# into baseline/_ref, where the reference-model GPU tests and
# `bench.py --impl reference` import it from.
#
# The reference checkout has no setup.py / pyproject.toml, so
# `pip install --target baseline/_ref <checkout>` refuses it.  This recipe
# copies the three packages the models import (layers, model, utils) to a
# temporary directory, adds a minimal pyproject.toml there (packaging only:
# no source file is changed) and pip-installs that copy offline into
# baseline/_ref.  baseline/_ref is git-ignored; it travels with the working
# tree to the GPU host.
#
# Usage: sh baseline/install_reference.sh <reference checkout>
set -eu
SRC=${1:?usage: install_reference.sh <reference checkout>}
HERE=$(cd "$(dirname "$0")" && pwd)
WORK=$(mktemp -d "${TMPDIR:-/tmp}/intp_reference.XXXXXX")
trap 'rm -rf "$WORK"' EXIT
cp -r "$SRC/layers" "$SRC/model" "$SRC/utils" "$WORK/"
find "$WORK" -name __pycache__ -type d -prune -exec rm -rf {} +
cat > "$WORK/pyproject.toml" <<'TOML'
[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "intp-preliminary-reference"
version = "0.0.0"

[tool.setuptools.packages.find]
include = ["layers*", "model*", "utils*"]
namespaces = true
TOML
rm -rf "$HERE/_ref"
python -m pip install --quiet --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --target "$HERE/_ref" "$WORK"
python - "$HERE/_ref" <<'PY'
import sys
sys.path.insert(0, sys.argv[1])
import model.deit_tiny_rot_hex_look, layers.mini_vit, utils.hex_graph  # noqa: F401
print("reference installed in", sys.argv[1])
PY
