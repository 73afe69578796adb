"""Configuration classes: the public configuration surface.

Parity: python/swiftllm/config.py (DataType, QuantizationMethod,
SchedulerPolicy, PreemptionMode :12-43; SamplingParams :46-145;
EngineConfig :148-245; ServerConfig :248-282; LoRARequest :285-301) and the
Rust mirror crates/swiftllm-core/src/config.rs. Where the Rust and Python
defaults disagree (prefix caching, chunked prefill, preemption mode) the
Python defaults win, as the Python API is the one users call.

Fields added for the B200 build: ``load_format`` ("auto" | "dummy"),
``comm_backend`` ("fused" | "nccl"), ``enforce_eager``,
``enable_cuda_graphs``, ``max_prefill_tokens``, ``watermark`` and
``SamplingParams.ignore_eos``. Every field can be overridden from the
environment as ``SWIFTLLM_<FIELD>`` (upper case).
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field, fields
from enum import Enum
from typing import Any, Dict, List, Optional


class DataType(Enum):
    FLOAT32 = "float32"
    FLOAT16 = "float16"
    BFLOAT16 = "bfloat16"
    INT8 = "int8"
    INT4 = "int4"
    FP8_E4M3 = "fp8_e4m3"
    FP8_E5M2 = "fp8_e5m2"
    AUTO = "auto"


class QuantizationMethod(Enum):
    NONE = "none"
    AWQ = "awq"
    GPTQ = "gptq"
    SQUEEZELLM = "squeezellm"
    GGUF = "gguf"
    FP8 = "fp8"
    INT8 = "int8"
    INT4 = "int4"
    NVFP4 = "nvfp4"


class SchedulerPolicy(Enum):
    FCFS = "fcfs"
    SJF = "sjf"
    PRIORITY = "priority"


class PreemptionMode(Enum):
    SWAP = "swap"
    RECOMPUTE = "recompute"


@dataclass
class SamplingParams:
    """Sampling and stopping parameters of one request.

    Stage order on the GPU and in the CPU oracle: repetition / frequency /
    presence penalties, temperature, min-p, top-k, top-p, draw. Greedy when
    ``temperature == 0`` or ``top_k == 1``.
    """

    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    min_p: float = 0.0
    max_tokens: int = 256
    min_tokens: int = 0
    stop: Optional[List[str]] = None
    stop_token_ids: Optional[List[int]] = None
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    repetition_penalty: float = 1.0
    seed: Optional[int] = None
    skip_special_tokens: bool = True
    include_stop_str_in_output: bool = False
    logprobs: Optional[int] = None
    prompt_logprobs: Optional[int] = None
    best_of: int = 1
    n: int = 1
    use_beam_search: bool = False
    length_penalty: float = 1.0
    early_stopping: bool = False
    ignore_eos: bool = False

    def __post_init__(self):
        if isinstance(self.stop, str):
            self.stop = [self.stop]
        if self.temperature < 0:
            raise ValueError(f"temperature must be non-negative, got {self.temperature}")
        if not 0 <= self.top_p <= 1:
            raise ValueError(f"top_p must be in [0, 1], got {self.top_p}")
        if self.top_k < -1 or self.top_k == 0:
            raise ValueError(f"top_k must be -1 (disabled) or >= 1, got {self.top_k}")
        if not 0 <= self.min_p <= 1:
            raise ValueError(f"min_p must be in [0, 1], got {self.min_p}")
        if self.max_tokens < 1:
            raise ValueError(f"max_tokens must be >= 1, got {self.max_tokens}")
        if self.min_tokens < 0 or self.min_tokens > self.max_tokens:
            raise ValueError(f"min_tokens must be in [0, max_tokens], got {self.min_tokens}")
        if self.n < 1:
            raise ValueError(f"n must be >= 1, got {self.n}")
        if self.best_of < self.n:
            if self.best_of == 1:
                self.best_of = self.n
            else:
                raise ValueError(
                    f"best_of must be >= n, got best_of={self.best_of}, n={self.n}")
        if self.use_beam_search and self.temperature != 0:
            raise ValueError("temperature must be 0 when using beam search")
        if self.logprobs is not None and self.logprobs < 0:
            raise ValueError(f"logprobs must be non-negative, got {self.logprobs}")
        if self.repetition_penalty <= 0:
            raise ValueError("repetition_penalty must be > 0")

    @property
    def is_greedy(self) -> bool:
        return self.temperature == 0 or self.top_k == 1

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "SamplingParams":
        return cls(**{k: v for k, v in d.items() if k in cls.__dataclass_fields__})

    def to_dict(self) -> Dict[str, Any]:
        return {f.name: getattr(self, f.name) for f in fields(self)}


def _env_override(obj) -> None:
    for f in fields(obj):
        key = "SWIFTLLM_" + f.name.upper()
        if key not in os.environ:
            continue
        raw = os.environ[key]
        cur = getattr(obj, f.name)
        if isinstance(cur, Enum):
            val: Any = type(cur)(raw)
        elif isinstance(cur, bool):
            val = raw.lower() in ("1", "true", "yes", "on")
        elif isinstance(cur, int):
            val = int(raw)
        elif isinstance(cur, float):
            val = float(raw)
        else:
            val = raw
        setattr(obj, f.name, val)


@dataclass
class EngineConfig:
    """Engine configuration (the Python API is the source of truth)."""

    model: str = ""
    tokenizer: Optional[str] = None
    dtype: DataType = DataType.AUTO
    quantization: QuantizationMethod = QuantizationMethod.NONE
    max_model_len: Optional[int] = None
    tensor_parallel_size: int = 1
    pipeline_parallel_size: int = 1
    gpu_memory_utilization: float = 0.90
    block_size: int = 16
    swap_space: float = 4.0
    max_num_seqs: int = 256
    max_num_batched_tokens: Optional[int] = None
    enable_prefix_caching: bool = False
    enable_chunked_prefill: bool = False
    max_paddings: int = 256
    scheduler_policy: SchedulerPolicy = SchedulerPolicy.FCFS
    preemption_mode: PreemptionMode = PreemptionMode.SWAP
    trust_remote_code: bool = False
    download_dir: Optional[str] = None
    seed: int = 0
    device: str = "auto"

    speculative_model: Optional[str] = None
    num_speculative_tokens: int = 5
    speculative_max_model_len: Optional[int] = None

    enable_lora: bool = False
    max_loras: int = 1
    max_lora_rank: int = 16
    lora_dtype: Optional[DataType] = None

    # B200 build additions
    load_format: str = "auto"
    comm_backend: str = "fused"
    enforce_eager: bool = False
    enable_cuda_graphs: bool = True
    max_prefill_tokens: int = 2048
    watermark: float = 0.01
    request_timeout_secs: float = 300.0
    num_gpu_blocks_override: Optional[int] = None

    def __post_init__(self):
        for name, enum in (("dtype", DataType), ("quantization", QuantizationMethod),
                           ("scheduler_policy", SchedulerPolicy),
                           ("preemption_mode", PreemptionMode)):
            v = getattr(self, name)
            if isinstance(v, str):
                setattr(self, name, enum(v))
            elif v is None and name == "quantization":
                self.quantization = QuantizationMethod.NONE
        _env_override(self)
        if self.gpu_memory_utilization <= 0 or self.gpu_memory_utilization > 1:
            raise ValueError(
                f"gpu_memory_utilization must be in (0, 1], got {self.gpu_memory_utilization}")
        if self.block_size not in (8, 16, 32):
            raise ValueError(f"block_size must be 8, 16, or 32, got {self.block_size}")
        if self.tensor_parallel_size < 1:
            raise ValueError(f"tensor_parallel_size must be >= 1, got {self.tensor_parallel_size}")
        if self.pipeline_parallel_size != 1:
            raise ValueError("pipeline_parallel_size > 1 is not supported; use tensor parallelism")
        if self.comm_backend not in ("fused", "nccl"):
            raise ValueError(f"comm_backend must be 'fused' or 'nccl', got {self.comm_backend}")
        if self.load_format not in ("auto", "dummy", "safetensors", "gguf", "pt"):
            raise ValueError(f"unknown load_format {self.load_format}")
        if self.max_num_seqs < 1:
            raise ValueError("max_num_seqs must be >= 1")
        if self.tokenizer is None:
            self.tokenizer = self.model

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "EngineConfig":
        return cls(**{k: v for k, v in d.items() if k in cls.__dataclass_fields__})

    def to_dict(self) -> Dict[str, Any]:
        out = {}
        for f in fields(self):
            v = getattr(self, f.name)
            out[f.name] = v.value if isinstance(v, Enum) else v
        return out


@dataclass
class ServerConfig:
    host: str = "0.0.0.0"
    port: int = 8000
    api_key: Optional[str] = None
    root_path: str = ""
    ssl_keyfile: Optional[str] = None
    ssl_certfile: Optional[str] = None
    cors_allow_origins: List[str] = field(default_factory=lambda: ["*"])
    max_log_len: Optional[int] = None
    response_role: str = "assistant"
    served_model_name: Optional[str] = None
    max_model_len_limit: Optional[int] = None
    max_num_seqs_limit: Optional[int] = None

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "ServerConfig":
        return cls(**{k: v for k, v in d.items() if k in cls.__dataclass_fields__})


@dataclass
class LoRARequest:
    """LoRA adapter request. Accepted and carried, not applied (the reference
    accepts it and never uses it either: python/swiftllm/engine.py:222)."""

    lora_name: str
    lora_path: str
    lora_local_path: Optional[str] = None

    @property
    def lora_int_id(self) -> int:
        return hash(self.lora_name) & 0xFFFFFFFF
