"""Logging setup. Level from ``SWIFTLLM_LOG`` (default WARNING); parity with
the reference's tracing subscriber level (crates/swiftllm-server/src/
main.rs:166-172, ``RUST_LOG`` / ``--log-level``)."""

from __future__ import annotations

import logging
import os

_configured = False


def get_logger(name: str) -> logging.Logger:
    global _configured
    if not _configured:
        level = os.environ.get("SWIFTLLM_LOG", os.environ.get("RUST_LOG", "WARNING")).upper()
        logging.basicConfig(level=getattr(logging, level, logging.WARNING),
                            format="%(asctime)s %(levelname)s %(name)s: %(message)s")
        _configured = True
    return logging.getLogger(name)


def set_level(level: str) -> None:
    logging.getLogger().setLevel(getattr(logging, level.upper(), logging.INFO))
