"""``swiftllm._core``: the low-level surface (RustEngine, RustScheduler, ...)."""

from swiftllm_b200.core_api import *  # noqa: F401,F403
