"""Standalone server launcher: ``swiftllm-server`` (console script) or
``python -m swiftllm_b200.server``.

Subcommands follow the reference's server binary
(crates/swiftllm-server/src/main.rs:37-150: serve / benchmark / convert /
info, the serve flag union: --model, --host, --port, --tensor-parallel-size,
--max-model-len, --gpu-memory-utilization, --block-size, --swap-space,
--enable-prefix-caching, --speculative-model, --num-speculative-tokens,
--api-key, --log-level, --trust-remote-code, --dtype). ``serve`` runs the
native C++ HTTP/1.1 + SSE front end (csrc/core/http_server.cpp) driving the
engine; a bare invocation with only flags means ``serve``.
"""

from __future__ import annotations

import sys
from typing import List, Optional

SUBCOMMANDS = ("serve", "benchmark", "convert", "info")


def main(argv: Optional[List[str]] = None) -> int:
    from ..cli import main as cli_main
    args = list(sys.argv[1:] if argv is None else argv)
    if not args or args[0] not in SUBCOMMANDS + ("-h", "--help"):
        args = ["serve"] + args
    return cli_main(args)


if __name__ == "__main__":
    sys.exit(main())
