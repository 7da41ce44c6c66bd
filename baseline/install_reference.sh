#!/usr/bin/env bash
# Install the unmodified reference implementation into baseline/_ref, where
# `bench.py --impl reference` and the planner-oracle tests import it from.
#
#   bash baseline/install_reference.sh <path-to-reference-checkout>
#
# The reference ships no packaging metadata (no setup.py / pyproject.toml), so pip
# refuses its directory as it is. The checkout is therefore copied to a scratch
# directory, a minimal pyproject.toml naming its `resihp` packages is added there, and
# pip installs that copy offline (no index, no build isolation, no dependencies: the
# reference needs only torch, which the image has). The installed Python files are the
# reference's own, byte for byte; the script checks that after the install.
set -euo pipefail

src=${1:?usage: install_reference.sh <path-to-reference-checkout>}
here=$(cd "$(dirname "$0")" && pwd)
dest="$here/_ref"
scratch=$(mktemp -d "${TMPDIR:-/tmp}/resihp_ref.XXXXXX")
trap 'rm -rf "$scratch"' EXIT

cp -r "$src/resihp" "$scratch/resihp"
cat > "$scratch/pyproject.toml" <<'TOML'
[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "resihp-reference"
version = "0.0.0"

[tool.setuptools.packages.find]
include = ["resihp*"]
TOML

rm -rf "$dest"
python -m pip install --quiet --no-index --no-build-isolation --no-deps \
    --find-links /opt/wheelhouse --target "$dest" "$scratch"

# Every installed module must equal the checkout's file.
status=0
while IFS= read -r f; do
    rel=${f#"$src/"}
    if ! cmp -s "$f" "$dest/$rel"; then
        echo "install_reference: $rel differs from the checkout" >&2
        status=1
    fi
done < <(find "$src/resihp" -name '*.py')
[ "$status" -eq 0 ] && echo "reference installed under $dest"
exit "$status"
