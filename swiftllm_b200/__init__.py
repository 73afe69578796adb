"""swiftllm_b200: a B200-native LLM inference and serving engine.

Public API parity with python/swiftllm/__init__.py:13-44 (LLM, AsyncLLM,
LLMEngine, RequestOutput, CompletionOutput, SamplingParams, EngineConfig,
ServerConfig, LoRARequest, resolve_model, SamplingStrategy, create_sampler).
"""

from .config import (DataType, EngineConfig, LoRARequest, PreemptionMode, QuantizationMethod,
                     SamplingParams, SchedulerPolicy, ServerConfig)
from .outputs import CompletionOutput, FinishReason, RequestOutput, TokenLogprob

__version__ = "0.1.0"

_LAZY = {
    "LLM": ("engine.llm", "LLM"),
    "AsyncLLM": ("engine.llm", "AsyncLLM"),
    "create_engine": ("engine.llm", "create_engine"),
    "generate": ("engine.llm", "generate"),
    "LLMEngine": ("engine.llm_engine", "LLMEngine"),
    "resolve_model": ("model_resolver", "resolve_model"),
    "SamplingStrategy": ("sampling", "SamplingStrategy"),
    "create_sampler": ("sampling", "create_sampler"),
}


def __getattr__(name):
    if name in _LAZY:
        import importlib
        mod, attr = _LAZY[name]
        return getattr(importlib.import_module(f".{mod}", __name__), attr)
    raise AttributeError(name)


def version() -> str:
    return __version__


__all__ = ["LLM", "AsyncLLM", "LLMEngine", "RequestOutput", "CompletionOutput", "SamplingParams",
           "EngineConfig", "ServerConfig", "LoRARequest", "resolve_model", "SamplingStrategy",
           "create_sampler", "FinishReason", "TokenLogprob", "DataType", "QuantizationMethod",
           "SchedulerPolicy", "PreemptionMode", "__version__"]
