#!/usr/bin/env bash
# Installs the unmodified reference (torchpp) into baseline/_ref for the GPU
# comparator (baseline/torchpp_gpu.py): its five CUDA extensions built for
# sm_100a against the CUTLASS headers vendored in the image, its Python
# package (plus torchpp/llmops, which pip skips), and a copy of its examples/LLM/fastqwen3.py model file (the
# package install does not carry examples).  Run in the build container,
# where the reference checkout exists; baseline/_ref is git-ignored and
# travels with the working tree to the GPU box.
#
#   bash baseline/install_ref.sh [REFERENCE_DIR]
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
REF="${1:-/root/reference}"
CUTLASS_INC="$(python -c 'import flashinfer, os; print(os.path.join(os.path.dirname(flashinfer.__file__), "data/cutlass/include"))')"
TMP="$(mktemp -d)"
cp -r "$REF" "$TMP/src"            # setup.py writes build/ into its source tree
CUDA_ARCH=100a CUTLASS_PATH="$CUTLASS_INC" MAX_JOBS="${MAX_JOBS:-8}" \
  python -m pip install --no-deps --no-index --no-build-isolation \
  --find-links /opt/wheelhouse --target "$HERE/_ref" "$TMP/src"
# torchpp/llmops has no __init__.py, so find_packages() skips it; the model
# file imports it (an implicit namespace package), so it is copied as is
cp -r "$REF/torchpp/llmops" "$HERE/_ref/torchpp/llmops"
mkdir -p "$HERE/_ref/examples/LLM"
cp "$REF/examples/LLM/fastqwen3.py" "$HERE/_ref/examples/LLM/fastqwen3.py"
rm -rf "$TMP"
