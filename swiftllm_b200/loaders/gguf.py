"""GGUF checkpoints: config from metadata and HF-named tensors.

Parity: crates/swiftllm-models/src/loaders/gguf.rs (architecture :266-275,
config from ``llama.*`` / ``phi.*`` keys :331-383). Block-quantised tensors
are dequantised to fp32 on the host by the C++ parser and then cast to the
model dtype (weights run as bf16 on the tensor cores).

llama.cpp's converter permutes the q / k projection rows from the HF
rotate-half layout to interleaved pairs; :func:`_unpermute` restores the
rotate-half order our RoPE kernel expects.
"""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from .. import _core
from ..models.config import ModelConfig


def _meta(f, key, default=None):
    md = f.metadata()
    return md.get(key, default)


def gguf_model_config(path: str) -> ModelConfig:
    f = _core.GgufFile(path)
    md = f.metadata()
    arch = md.get("general.architecture", "llama")
    fam = {"llama": "llama", "mistral": "mistral", "qwen2": "qwen2", "phi2": "phi"}.get(arch, "llama")
    p = arch
    h = int(md.get(f"{p}.embedding_length", 4096))
    nh = int(md.get(f"{p}.attention.head_count", 32))
    nkv = int(md.get(f"{p}.attention.head_count_kv", nh))
    vocab = md.get(f"{p}.vocab_size")
    if vocab is None:
        toks = md.get("tokenizer.ggml.tokens")
        vocab = len(toks) if toks is not None else 32000
    inter = int(md.get(f"{p}.feed_forward_length", 4 * h))
    cfg = ModelConfig(
        architecture=fam, hidden_size=h, intermediate_size=inter,
        num_layers=int(md.get(f"{p}.block_count", 32)), num_heads=nh, num_kv_heads=nkv,
        head_dim=h // nh, vocab_size=int(vocab),
        rms_norm_eps=float(md.get(f"{p}.attention.layer_norm_rms_epsilon",
                                  md.get(f"{p}.attention.layer_norm_epsilon", 1e-5))),
        rope_theta=float(md.get(f"{p}.rope.freq_base", 10000.0)),
        max_position_embeddings=int(md.get(f"{p}.context_length", 4096)),
        bos_token_id=int(md.get("tokenizer.ggml.bos_token_id", 1)),
        eos_token_id=int(md.get("tokenizer.ggml.eos_token_id", 2)),
        num_experts=int(md.get(f"{p}.expert_count", 0)),
        num_experts_per_tok=int(md.get(f"{p}.expert_used_count", 0)),
    )
    if cfg.num_experts:
        cfg.architecture = "mixtral"
    cfg.name = str(md.get("general.name", "gguf"))
    return cfg


def _unpermute(w: torch.Tensor, n_head: int) -> torch.Tensor:
    """Inverse of llama.cpp's q/k row permutation (interleaved -> rotate-half)."""
    rows = w.shape[0]
    return (w.reshape(n_head, rows // n_head // 2, 2, *w.shape[1:])
            .transpose(1, 2).reshape(w.shape))


_LAYER_MAP = {
    "attn_norm.weight": "input_layernorm.weight",
    "attn_q.weight": "self_attn.q_proj.weight",
    "attn_k.weight": "self_attn.k_proj.weight",
    "attn_v.weight": "self_attn.v_proj.weight",
    "attn_q.bias": "self_attn.q_proj.bias",
    "attn_k.bias": "self_attn.k_proj.bias",
    "attn_v.bias": "self_attn.v_proj.bias",
    "attn_output.weight": "self_attn.o_proj.weight",
    "ffn_norm.weight": "post_attention_layernorm.weight",
    "ffn_gate.weight": "mlp.gate_proj.weight",
    "ffn_up.weight": "mlp.up_proj.weight",
    "ffn_down.weight": "mlp.down_proj.weight",
    "ffn_gate_inp.weight": "block_sparse_moe.gate.weight",
}


class GgufCheckpoint:
    def __init__(self, path: str):
        self.f = _core.GgufFile(path)
        self.cfg = gguf_model_config(path)
        self.names = {}
        for info in self.f.tensor_infos():
            n = info["name"]
            hf = self._hf_name(n)
            if hf:
                self.names[hf] = n

    def _hf_name(self, n: str) -> Optional[str]:
        if n == "token_embd.weight":
            return "model.embed_tokens.weight"
        if n == "output_norm.weight":
            return "model.norm.weight"
        if n == "output.weight":
            return "lm_head.weight"
        if n.startswith("blk."):
            _, i, rest = n.split(".", 2)
            if rest in _LAYER_MAP:
                return f"model.layers.{i}.{_LAYER_MAP[rest]}"
            for e_key, w in (("ffn_gate_exps.weight", "w1"), ("ffn_up_exps.weight", "w3"),
                             ("ffn_down_exps.weight", "w2")):
                if rest == e_key:
                    return f"model.layers.{i}.experts_packed.{w}"
        return None

    def keys(self):
        return list(self.names)

    def get(self, name: str) -> Optional[torch.Tensor]:
        if ".block_sparse_moe.experts." in name:
            # model.layers.{i}.block_sparse_moe.experts.{e}.w1.weight
            parts = name.split(".")
            i, e, w = parts[2], int(parts[5]), parts[6]
            packed = self.get(f"model.layers.{i}.experts_packed.{w}")
            return None if packed is None else packed[e]
        g = self.names.get(name)
        if g is None:
            return None
        t = torch.from_numpy(self.f.dequant(g))
        if name.endswith("q_proj.weight"):
            t = _unpermute(t, self.cfg.num_heads)
        elif name.endswith("k_proj.weight"):
            t = _unpermute(t, self.cfg.num_kv_heads)
        return t
