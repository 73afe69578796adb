"""Request output types.

Parity: python/swiftllm/engine.py:29-99 (FinishReason, TokenLogprob,
CompletionOutput, RequestOutput) and the Rust RequestOutput /
RequestMetrics (crates/swiftllm-core/src/types.rs:449-529).
``RequestOutput.metrics`` carries arrival, first_scheduled, first_token,
finished, ttft, tpot, prompt_tokens and completion_tokens (seconds, from the
engine's monotonic clock).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from typing import Dict, List, Optional, Union


class FinishReason(Enum):
    STOP = "stop"
    LENGTH = "length"
    ABORT = "abort"


@dataclass
class TokenLogprob:
    token_id: int
    token: str
    logprob: float
    bytes: Optional[List[int]] = None


@dataclass
class CompletionOutput:
    index: int
    text: str
    token_ids: List[int] = field(default_factory=list)
    cumulative_logprob: Optional[float] = None
    logprobs: Optional[List[TokenLogprob]] = None
    finish_reason: Optional[FinishReason] = None
    stop_reason: Optional[Union[int, str]] = None

    @property
    def finished(self) -> bool:
        return self.finish_reason is not None


@dataclass
class RequestOutput:
    request_id: str
    prompt: Optional[str]
    prompt_token_ids: List[int]
    prompt_logprobs: Optional[List[TokenLogprob]] = None
    outputs: List[CompletionOutput] = field(default_factory=list)
    finished: bool = False
    metrics: Optional[Dict[str, float]] = None

    def __repr__(self) -> str:
        p = self.prompt
        if p and len(p) > 50:
            p = p[:50] + "..."
        return (f"RequestOutput(request_id={self.request_id!r}, prompt={p!r}, "
                f"num_outputs={len(self.outputs)}, finished={self.finished})")
