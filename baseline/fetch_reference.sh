#!/bin/sh
# Puts an unmodified copy of the NEED reference's Python sources and licence
# under baseline/_ref/ (git-ignored, never committed; it travels with the
# working tree the way the built library does).  The reference has no
# setup.py or pyproject.toml, so `pip install --target baseline/_ref` refuses
# it; a plain copy is the install.  Source: $NEED_REFERENCE, default
# /root/reference.  Only tests/test_model_gpu.py, tests/golden/make_golden.py
# and bench.py's reference GPU bars import it, and each says so when it is
# absent.
set -eu
src="${NEED_REFERENCE:-/root/reference}"
dst="$(dirname "$0")/_ref"
mkdir -p "$dst"
cp "$src"/*.py "$src"/LICENSE "$dst"/
echo "copied $(ls "$dst" | wc -l) files from $src to $dst"
