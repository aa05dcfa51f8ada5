#!/usr/bin/env bash
# Copies the reference's kernel package, its attention layer and its kernel tests, unmodified, into baseline/_ref/
# (git-ignored) so that the comparator test and the bench's `reference_gpu` side object can run the reference's OWN
# GPU kernels next to this package's on the same inputs:
#   diffulex_kernel/                     Triton store / load kernels, TileLang decode / prefill kernels, wrappers
#   diffulex/attention/                  Attention layer + metadata base (no diffulex/__init__.py: the directory is
#                                        then a namespace package and importing it does not start the engine)
#   diffulex/strategy/*/attention/metadata.py   the two strategies' metadata dataclasses
#   tests/python/kernel/                 the reference's kernel tests (naive checks), as ref_tests/
# Usage: baseline/make_ref.sh /path/to/Diffulex
set -euo pipefail
src="${1:?path of the reference checkout}"
here="$(cd "$(dirname "$0")" && pwd)"
dst="$here/_ref"
mkdir -p "$dst/diffulex/strategy/d2f/attention" "$dst/diffulex/strategy/block_diffusion/attention" "$dst/ref_tests"
cp -r "$src/diffulex_kernel" "$dst/"
cp -r "$src/diffulex/attention" "$dst/diffulex/"
cp "$src/diffulex/strategy/d2f/attention/metadata.py" "$dst/diffulex/strategy/d2f/attention/"
cp "$src/diffulex/strategy/block_diffusion/attention/metadata.py" "$dst/diffulex/strategy/block_diffusion/attention/"
cp "$src"/tests/python/kernel/*.py "$dst/ref_tests/"
find "$dst" -name __pycache__ -type d -prune -exec rm -r {} +
echo "reference copied to $dst"
