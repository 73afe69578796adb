"""Model configuration: HF ``config.json`` parsing, architecture detection
and named presets for random-init (``load_format="dummy"``) runs.

Parity: crates/swiftllm-models/src/lib.rs:18-130 (ModelConfig, GQA helpers,
kv_cache_size_per_token), crates/swiftllm-models/src/loaders/huggingface.rs
(HfConfig defaults :16-123, detect_architecture :146-211, convert_hf_config
:214-260), crates/swiftllm-core/src/config.rs:118-149 (architecture list) and
:218-242 (RoPE scaling types).
"""

from __future__ import annotations

import json
import os
from dataclasses import asdict, dataclass, field
from typing import Any, Dict, Optional

ARCHITECTURES = {
    # HF class name / model_type -> internal family
    "LlamaForCausalLM": "llama", "llama": "llama",
    "MistralForCausalLM": "mistral", "mistral": "mistral",
    "MixtralForCausalLM": "mixtral", "mixtral": "mixtral",
    "Qwen2ForCausalLM": "qwen2", "qwen2": "qwen2", "QWenLMHeadModel": "qwen2", "qwen": "qwen2",
    "PhiForCausalLM": "phi", "phi": "phi",
    "Phi3ForCausalLM": "phi3", "phi3": "phi3",
}


@dataclass
class ModelConfig:
    architecture: str = "llama"
    hidden_size: int = 4096
    intermediate_size: int = 11008
    num_layers: int = 32
    num_heads: int = 32
    num_kv_heads: int = 32
    head_dim: int = 128
    vocab_size: int = 32000
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    rope_scaling: Optional[Dict[str, Any]] = None
    partial_rotary_factor: float = 1.0
    max_position_embeddings: int = 4096
    tie_word_embeddings: bool = False
    attention_bias: bool = False       # qkv bias (Qwen2)
    mlp_bias: bool = False
    sliding_window: Optional[int] = None
    num_experts: int = 0
    num_experts_per_tok: int = 0
    hidden_act: str = "silu"
    norm_type: str = "rmsnorm"         # "rmsnorm" | "layernorm" (Phi)
    parallel_block: bool = False       # Phi: attention and MLP read the same input
    position_embedding: str = "rope"   # "rope" | "alibi" (per-head linear score bias, no RoPE)
    bos_token_id: int = 1
    eos_token_id: int = 2
    name: str = ""

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def num_queries_per_kv(self) -> int:
        return self.num_heads // self.num_kv_heads

    @property
    def is_gqa(self) -> bool:
        return 1 < self.num_kv_heads < self.num_heads

    @property
    def is_mqa(self) -> bool:
        return self.num_kv_heads == 1

    @property
    def rotary_dim(self) -> int:
        if self.position_embedding == "alibi":
            return 0
        return int(self.head_dim * self.partial_rotary_factor)

    def kv_cache_bytes_per_token(self, dtype_bytes: int = 2) -> int:
        return 2 * self.num_layers * self.num_kv_heads * self.head_dim * dtype_bytes

    def num_params(self) -> int:
        h, i, v = self.hidden_size, self.intermediate_size, self.vocab_size
        attn = h * (self.q_size + 2 * self.kv_size) + self.q_size * h
        n_mlp = max(self.num_experts, 1)
        mlp = n_mlp * 3 * h * i + (h * self.num_experts if self.num_experts else 0)
        emb = v * h * (1 if self.tie_word_embeddings else 2)
        return self.num_layers * (attn + mlp + 2 * h) + emb + h

    def to_dict(self) -> Dict[str, Any]:
        return asdict(self)


PRESETS: Dict[str, ModelConfig] = {
    # tiny LLaMA for the CPU oracle
    "tiny-llama": ModelConfig(architecture="llama", hidden_size=256, intermediate_size=688,
                              num_layers=2, num_heads=4, num_kv_heads=2, head_dim=64,
                              vocab_size=32000, rms_norm_eps=1e-5, rope_theta=10000.0,
                              max_position_embeddings=2048),
    # the tiny LLaMA with ALiBi instead of RoPE (kernel / engine coverage)
    "tiny-llama-alibi": ModelConfig(architecture="llama", hidden_size=256, intermediate_size=688,
                                    num_layers=2, num_heads=4, num_kv_heads=2, head_dim=64,
                                    vocab_size=32000, rms_norm_eps=1e-5, position_embedding="alibi",
                                    max_position_embeddings=2048),
    "llama-2-7b": ModelConfig(architecture="llama", hidden_size=4096, intermediate_size=11008,
                              num_layers=32, num_heads=32, num_kv_heads=32, head_dim=128,
                              vocab_size=32000, rope_theta=10000.0, max_position_embeddings=4096),
    "llama-2-13b": ModelConfig(architecture="llama", hidden_size=5120, intermediate_size=13824,
                               num_layers=40, num_heads=40, num_kv_heads=40, head_dim=128,
                               vocab_size=32000, max_position_embeddings=4096),
    "llama-3-8b": ModelConfig(architecture="llama", hidden_size=4096, intermediate_size=14336,
                              num_layers=32, num_heads=32, num_kv_heads=8, head_dim=128,
                              vocab_size=128256, rope_theta=500000.0, max_position_embeddings=8192,
                              bos_token_id=128000, eos_token_id=128001),
    "llama-3-70b": ModelConfig(architecture="llama", hidden_size=8192, intermediate_size=28672,
                               num_layers=80, num_heads=64, num_kv_heads=8, head_dim=128,
                               vocab_size=128256, rope_theta=500000.0, max_position_embeddings=8192,
                               bos_token_id=128000, eos_token_id=128001),
    "mistral-7b": ModelConfig(architecture="mistral", hidden_size=4096, intermediate_size=14336,
                              num_layers=32, num_heads=32, num_kv_heads=8, head_dim=128,
                              vocab_size=32000, rope_theta=10000.0, sliding_window=4096,
                              max_position_embeddings=32768),
    "mixtral-8x7b": ModelConfig(architecture="mixtral", hidden_size=4096, intermediate_size=14336,
                                num_layers=32, num_heads=32, num_kv_heads=8, head_dim=128,
                                vocab_size=32000, rope_theta=1e6, num_experts=8,
                                num_experts_per_tok=2, max_position_embeddings=32768),
    "tiny-mixtral": ModelConfig(architecture="mixtral", hidden_size=256, intermediate_size=512,
                                num_layers=2, num_heads=4, num_kv_heads=2, head_dim=64,
                                vocab_size=1024, num_experts=4, num_experts_per_tok=2,
                                max_position_embeddings=2048),
    "qwen2-7b": ModelConfig(architecture="qwen2", hidden_size=3584, intermediate_size=18944,
                            num_layers=28, num_heads=28, num_kv_heads=4, head_dim=128,
                            vocab_size=152064, rope_theta=1e6, attention_bias=True,
                            rms_norm_eps=1e-6, max_position_embeddings=32768),
    "tiny-qwen2": ModelConfig(architecture="qwen2", hidden_size=256, intermediate_size=512,
                              num_layers=2, num_heads=4, num_kv_heads=2, head_dim=64,
                              vocab_size=1024, attention_bias=True, rms_norm_eps=1e-6,
                              max_position_embeddings=2048),
    "phi-2": ModelConfig(architecture="phi", hidden_size=2560, intermediate_size=10240,
                         num_layers=32, num_heads=32, num_kv_heads=32, head_dim=80,
                         vocab_size=51200, partial_rotary_factor=0.4, hidden_act="gelu_new",
                         norm_type="layernorm", parallel_block=True, attention_bias=True,
                         mlp_bias=True, rms_norm_eps=1e-5, max_position_embeddings=2048),
    "tiny-phi": ModelConfig(architecture="phi", hidden_size=256, intermediate_size=1024,
                            num_layers=2, num_heads=4, num_kv_heads=4, head_dim=64,
                            vocab_size=1024, partial_rotary_factor=0.5, hidden_act="gelu_new",
                            norm_type="layernorm", parallel_block=True, attention_bias=True,
                            mlp_bias=True, max_position_embeddings=2048),
}
for _k, _v in PRESETS.items():
    _v.name = _k


def detect_architecture(hf: Dict[str, Any]) -> str:
    for a in hf.get("architectures") or []:
        if a in ARCHITECTURES:
            return ARCHITECTURES[a]
    mt = hf.get("model_type", "")
    if mt in ARCHITECTURES:
        return ARCHITECTURES[mt]
    raise ValueError(f"unsupported architecture: {hf.get('architectures')} / {mt!r}")


def from_hf_config(hf: Dict[str, Any]) -> ModelConfig:
    arch = detect_architecture(hf)
    h = int(hf.get("hidden_size", hf.get("n_embd", 4096)))
    nh = int(hf.get("num_attention_heads", hf.get("n_head", 32)))
    nkv = int(hf.get("num_key_value_heads") or nh)
    head_dim = int(hf.get("head_dim") or h // nh)
    inter = hf.get("intermediate_size") or hf.get("n_inner")
    if not inter:
        # SwiGLU default: 8H/3 rounded up to a multiple of 256
        inter = ((8 * h // 3) + 255) // 256 * 256 if arch != "phi" else 4 * h
    eos = hf.get("eos_token_id", 2)
    if isinstance(eos, list):
        eos = eos[0]
    cfg = ModelConfig(
        architecture=arch,
        hidden_size=h,
        intermediate_size=int(inter),
        num_layers=int(hf.get("num_hidden_layers", hf.get("n_layer", 32))),
        num_heads=nh,
        num_kv_heads=nkv,
        head_dim=head_dim,
        vocab_size=int(hf.get("vocab_size", 32000)),
        rms_norm_eps=float(hf.get("rms_norm_eps", hf.get("layer_norm_eps",
                                                          hf.get("layer_norm_epsilon", 1e-5)))),
        rope_theta=float(hf.get("rope_theta", 10000.0)),
        rope_scaling=hf.get("rope_scaling"),
        partial_rotary_factor=float(hf.get("partial_rotary_factor", 1.0)),
        max_position_embeddings=int(hf.get("max_position_embeddings", 4096)),
        tie_word_embeddings=bool(hf.get("tie_word_embeddings", False)),
        attention_bias=bool(hf.get("attention_bias", arch in ("qwen2", "phi"))),
        mlp_bias=bool(hf.get("mlp_bias", arch == "phi")),
        sliding_window=hf.get("sliding_window") if hf.get("use_sliding_window", True) else None,
        num_experts=int(hf.get("num_local_experts", 0)),
        num_experts_per_tok=int(hf.get("num_experts_per_tok", 0)),
        hidden_act=hf.get("hidden_act", hf.get("activation_function", "silu")),
        norm_type="layernorm" if arch == "phi" else "rmsnorm",
        parallel_block=arch == "phi",
        bos_token_id=int(hf.get("bos_token_id") or 1),
        eos_token_id=int(eos if eos is not None else 2),
    )
    if arch == "llama" or arch == "qwen2":
        cfg.sliding_window = None
    return cfg


def load_config(model: str) -> ModelConfig:
    """Model config from a preset name, a directory with config.json, a
    config.json path, or a GGUF file."""
    key = model.lower()
    if key.startswith("dummy:"):
        key = key[len("dummy:"):]
    if key in PRESETS:
        return ModelConfig(**PRESETS[key].to_dict())
    if os.path.isdir(model) and os.path.exists(os.path.join(model, "config.json")):
        with open(os.path.join(model, "config.json")) as f:
            cfg = from_hf_config(json.load(f))
        cfg.name = os.path.basename(os.path.normpath(model))
        return cfg
    if model.endswith(".json") and os.path.exists(model):
        with open(model) as f:
            return from_hf_config(json.load(f))
    if model.lower().endswith(".gguf") and os.path.exists(model):
        from ..loaders.gguf import gguf_model_config
        return gguf_model_config(model)
    raise ValueError(f"cannot resolve a model config for {model!r} "
                     f"(presets: {', '.join(sorted(PRESETS))})")
