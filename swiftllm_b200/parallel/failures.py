"""Failure taxonomy of the distributed runtime (host side).

Parity: crates/swiftllm-core/src/error.rs (Error variants and the
is_oom / is_timeout / is_cancelled predicates :157-170). Device-side waits
in the fused communication kernels report through a status word instead of
trapping; the host turns a non-zero word into :class:`CommTimeoutError`.
"""


class SwiftError(RuntimeError):
    pass


class WorkerDiedError(SwiftError):
    """A tensor-parallel worker process exited or stopped heartbeating."""


class CommTimeoutError(SwiftError, TimeoutError):
    """A bounded wait on a peer (flag, barrier, channel) ran out."""


class OutOfBlocksError(SwiftError):
    """The KV pool cannot hold the request even after preemption."""


def is_timeout(e: BaseException) -> bool:
    return isinstance(e, TimeoutError)


def is_oom(e: BaseException) -> bool:
    return isinstance(e, (OutOfBlocksError, MemoryError)) or "out of memory" in str(e).lower()


def is_cancelled(e: BaseException) -> bool:
    import asyncio
    return isinstance(e, asyncio.CancelledError)
