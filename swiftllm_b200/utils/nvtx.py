"""NVTX ranges per engine phase (schedule / prepare / forward / sample).
Enabled with ``SWIFTLLM_NVTX=1``; free otherwise."""

from __future__ import annotations

import contextlib
import os

_ENABLED = os.environ.get("SWIFTLLM_NVTX", "0") == "1"


@contextlib.contextmanager
def _nvtx(name: str):
    import torch
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def range(name: str):  # noqa: A001 - mirrors nvtx naming
    if _ENABLED:
        return _nvtx(name)
    return contextlib.nullcontext()
