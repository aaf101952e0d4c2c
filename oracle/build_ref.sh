#!/usr/bin/env bash
# Builds oracle/_ref: the unmodified reference compiler (garrick247/opencuda,
# pure Python) installed from its own sources so that it can run as the live
# oracle and as the timed CPU baseline on a machine without the reference
# checkout.  The reference is read-only, so setuptools builds from a copy in
# a temporary directory.  Output goes only to oracle/_ref (git-ignored).
#
# usage: oracle/build_ref.sh [REFERENCE_DIR]
#   REFERENCE_DIR defaults to $OCB_REFERENCE_DIR, else /root/reference (the
#   read-only checkout on the build machine).  Without a checkout there it
#   keeps the existing install and exits 0.
set -euo pipefail
REF="${1:-${OCB_REFERENCE_DIR:-/root/reference}}"
HERE="$(cd "$(dirname "$0")" && pwd)"
OUT="$HERE/_ref/py"
if [ ! -f "$REF/opencuda/frontend/lexer.py" ]; then
    echo "build_ref: no reference at $REF; keeping existing $OUT" >&2
    exit 0
fi
TMP="$(mktemp -d)"
trap 'rm -rf "$TMP"' EXIT
cp -r "$REF/opencuda" "$REF/pyproject.toml" "$TMP/"
rm -rf "$OUT"
mkdir -p "$HERE/_ref"
python -m pip install --quiet --no-index --no-build-isolation --no-deps \
    --find-links /opt/wheelhouse --target "$OUT" "$TMP"
# Byte-compile so that worker start-up on the GPU host stays short.
python -m compileall -q "$OUT/opencuda" >/dev/null
echo "build_ref: installed reference into $OUT"
