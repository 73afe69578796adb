"""Test configuration: the ``gpu`` marker, and an in-tree build of the CPU
core extension when it is missing (the CUDA extension is built by
``python setup.py build_ext --inplace`` / ``__graft_entry__.build()``)."""

import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")
    config.addinivalue_line("markers", "slow: long-running test")
    import glob
    if not glob.glob(os.path.join(ROOT, "swiftllm_b200", "_core*.so")):
        env = dict(os.environ, SWIFTLLM_BUILD="core", MAX_JOBS="8")
        subprocess.run([sys.executable, "setup.py", "build_ext", "--inplace"], cwd=ROOT,
                       env=env, check=True, stdout=subprocess.DEVNULL)


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
