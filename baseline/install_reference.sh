#!/usr/bin/env bash
# Installs the unmodified reference package (extended_einsum, pure Python) into
# baseline/_ref for `bench.py --impl reference` and the drop-in tests.
#
# The reference's pyproject names the `uv_build` backend, which is not in the
# offline wheelhouse, so the package is built from a copy under /tmp whose
# [build-system] table alone is switched to setuptools (same package, same
# src/ layout; no source file is touched).  Its dependencies (numpy, torch)
# are already installed; sesum is absent and only needed off this path, hence
# --no-deps.
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
src="${1:-/root/reference}"
tmp="$(mktemp -d /tmp/xe_ref_build.XXXXXX)"
cp -r "$src"/. "$tmp"/
python - "$tmp/pyproject.toml" <<'PY'
import re, sys
path = sys.argv[1]
text = open(path).read()
text = re.sub(r"\[build-system\][^\[]*",
              '[build-system]\nrequires = ["setuptools"]\nbuild-backend = "setuptools.build_meta"\n\n'
              '[tool.setuptools.packages.find]\nwhere = ["src"]\n\n'
              '[tool.setuptools.package-data]\n"*" = ["py.typed"]\n\n', text, count=1)
open(path, "w").write(text)
PY
rm -rf "$here/_ref"
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse --target "$here/_ref" "$tmp"
rm -rf "$tmp"
python -c "import sys; sys.path.insert(0, '$here/_ref'); import extended_einsum, os; print('installed', os.path.dirname(extended_einsum.__file__))"
