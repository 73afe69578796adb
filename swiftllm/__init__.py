"""Drop-in import name: ``import swiftllm`` resolves to the B200 build."""

import sys as _sys

import swiftllm_b200 as _impl
from swiftllm_b200 import *  # noqa: F401,F403
from swiftllm_b200 import __version__  # noqa: F401


def __getattr__(name):
    return getattr(_impl, name)
import importlib as _importlib  # noqa: E402

# the reference's low-level surface; imported explicitly because the module
# __getattr__ above would otherwise answer ``_core`` with the C++ extension
_core = _importlib.import_module(__name__ + "._core")
