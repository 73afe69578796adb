#!/usr/bin/env bash
# Build swiftllm_b200 in place and check the install.
#
#   ./install.sh            # C++ core + sm_100a CUDA kernels, then import checks
#   ./install.sh --cpu      # C++ core only (no nvcc needed; CPU paths and tests)
#   ./install.sh --test     # also run the CPU test suite
#
# Needs: Python >= 3.10 with torch, pybind11 and ninja importable; g++ with
# C++17; for the kernels, nvcc >= 12.8 (sm_100a). The extensions are built
# in the source tree (swiftllm_b200/_core*.so, swiftllm_b200/_C*.so), so the
# checkout can be used directly (add it to PYTHONPATH) or installed with
# `pip install --no-build-isolation -e .`.
set -euo pipefail
cd "$(dirname "$0")"
PY=${PYTHON:-python3}
WHAT=all
TEST=0
for a in "$@"; do
  case "$a" in
    --cpu) WHAT=core ;;
    --test) TEST=1 ;;
    -h|--help) sed -n '2,12p' "$0"; exit 0 ;;
    *) echo "unknown option $a" >&2; exit 2 ;;
  esac
done

"$PY" - <<'PYEOF'
import sys
assert sys.version_info >= (3, 10), f"Python >= 3.10 needed, found {sys.version.split()[0]}"
for m in ("torch", "pybind11", "ninja", "numpy"):
    __import__(m)
import torch
print(f"python {sys.version.split()[0]}, torch {torch.__version__}, cuda available: {torch.cuda.is_available()}")
PYEOF

if [ "$WHAT" = all ]; then
  command -v nvcc >/dev/null || { echo "nvcc not found (use --cpu for the C++ core only)" >&2; exit 1; }
  nvcc --version | tail -n 1
fi

SWIFTLLM_BUILD=$WHAT MAX_JOBS=${MAX_JOBS:-8} "$PY" setup.py build_ext --inplace

"$PY" - "$WHAT" <<'PYEOF'
import sys
import torch  # noqa: F401  (libtorch before the extensions)
import swiftllm_b200
from swiftllm_b200 import _core  # noqa: F401
if sys.argv[1] == "all":
    from swiftllm_b200 import _C  # noqa: F401
    print("kernels: swiftllm_b200._C loaded")
print("swiftllm_b200", swiftllm_b200.__version__, "ready")
PYEOF

if [ "$TEST" = 1 ]; then
  "$PY" -m pytest tests -q -m "not gpu"
fi
