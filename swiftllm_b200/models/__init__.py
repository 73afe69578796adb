"""Model families and configuration (Llama 2/3, Mistral, Qwen2, Mixtral, Phi).

Parity: crates/swiftllm-models/src/architectures/mod.rs (TransformerModel +
create_model :23-77; the reference rejects Mixtral, this build supports it).
"""

from .config import ModelConfig, PRESETS, detect_architecture, from_hf_config, load_config

SUPPORTED_ARCHITECTURES = ("llama", "mistral", "qwen2", "mixtral", "phi")


def create_model(cfg, dtype, device, tp=None, max_pos=None):
    from .decoder import DecoderModel
    if cfg.architecture not in SUPPORTED_ARCHITECTURES:
        raise ValueError(f"unsupported architecture {cfg.architecture!r}")
    return DecoderModel(cfg, dtype, device, tp, max_pos)
