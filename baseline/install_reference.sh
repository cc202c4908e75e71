#!/usr/bin/env bash
# Install the reference (lmjlmj1234/mini-vllm-continuous-batching-lab, pure
# Python) into baseline/_ref, offline, from a checkout of it.  The reference
# engine runs from there for the config-5 drop-in test and for timing the
# reference's own CPU path.  The build writes into its source tree, so it
# builds from a copy.
#   usage: baseline/install_reference.sh <path to the reference checkout>
set -euo pipefail
src="${1:?path to the reference checkout}"
here="$(cd "$(dirname "$0")" && pwd)"
tmp="$(mktemp -d)"
cp -r "$src" "$tmp/ref"
python -m pip install --no-index --no-build-isolation --find-links /opt/wheelhouse \
    --target "$here/_ref" --no-deps "$tmp/ref"
rm -rf "$tmp"
