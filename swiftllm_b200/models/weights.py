"""HF checkpoint name mapping and per-rank sharded loading.

Parity: crates/swiftllm-models/src/loaders/mod.rs:84-136 (WeightMapper
renames for Qwen / Phi) and crates/swiftllm-core/src/execution/
tensor_parallel.rs:162-202 (shard_tensor ranges). Each full tensor is read
(a zero-copy view of the mmap'd checkpoint), the rank's rows or columns are
sliced, and only that slice is copied to the device.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch


def _copy(dst: torch.Tensor, src: torch.Tensor, name: str) -> None:
    if tuple(dst.shape) != tuple(src.shape):
        raise ValueError(f"{name}: checkpoint shape {tuple(src.shape)} != expected {tuple(dst.shape)}")
    dst.copy_(src.to(dst.dtype), non_blocking=False)


def load_hf_weights(model, get: Callable[[str], Optional[torch.Tensor]]) -> None:
    c = model.cfg
    D = c.head_dim
    r = model.tp.rank
    qh, kvh = model.local_heads, model.local_kv_heads
    q0, k0 = r * qh * D, model.kv_head_start * D
    I0, In = r * model.local_inter, model.local_inter
    phi = c.architecture == "phi"

    def need(name):
        t = get(name)
        if t is None:
            raise KeyError(f"checkpoint is missing {name}")
        return t

    _copy(model.embed, need("model.embed_tokens.weight")[model.vocab_start:model.vocab_end], "embed")
    for i, L in enumerate(model.layers):
        p = f"model.layers.{i}."
        _copy(L.ln1, need(p + "input_layernorm.weight"), "ln1")
        if L.ln1_b is not None:
            _copy(L.ln1_b, need(p + "input_layernorm.bias"), "ln1_b")
        wq = need(p + "self_attn.q_proj.weight")[q0:q0 + qh * D]
        wk = need(p + "self_attn.k_proj.weight")[k0:k0 + kvh * D]
        wv = need(p + "self_attn.v_proj.weight")[k0:k0 + kvh * D]
        _copy(L.wqkv, torch.cat([wq, wk, wv], 0), f"{p}qkv")
        if L.bqkv is not None:
            bq = need(p + "self_attn.q_proj.bias")[q0:q0 + qh * D]
            bk = need(p + "self_attn.k_proj.bias")[k0:k0 + kvh * D]
            bv = need(p + "self_attn.v_proj.bias")[k0:k0 + kvh * D]
            _copy(L.bqkv, torch.cat([bq, bk, bv], 0), f"{p}qkv.bias")
        o_name = p + ("self_attn.dense" if phi else "self_attn.o_proj")
        _copy(L.wo, need(o_name + ".weight")[:, q0:q0 + qh * D], o_name)
        if L.bo is not None:
            _copy(L.bo, need(o_name + ".bias"), o_name + ".bias")
        if hasattr(L, "ln2"):
            _copy(L.ln2, need(p + "post_attention_layernorm.weight"), "ln2")
        if c.num_experts:
            fused = get(p + "mlp.experts.gate_up_proj")  # transformers >= 5 layout
            if fused is not None:
                _copy(L.router, need(p + "mlp.gate.weight"), "router")
                Ifull = c.intermediate_size
                mi0, mi = (0, Ifull) if model.ep else (I0, In)
                sl = slice(model.e0, model.e0 + model.e_local)
                gu = fused[sl]
                _copy(L.w13, torch.cat([gu[:, mi0:mi0 + mi], gu[:, Ifull + mi0:Ifull + mi0 + mi]], 1), "w13")
                _copy(L.w2, need(p + "mlp.experts.down_proj")[sl][:, :, mi0:mi0 + mi], "w2")
                continue
            _copy(L.router, need(p + "block_sparse_moe.gate.weight"), "router")
            mi0, mi = (0, c.intermediate_size) if model.ep else (I0, In)
            for le in range(model.e_local):
                q = p + f"block_sparse_moe.experts.{model.e0 + le}."
                g = need(q + "w1.weight")[mi0:mi0 + mi]
                u = need(q + "w3.weight")[mi0:mi0 + mi]
                _copy(L.w13[le], torch.cat([g, u], 0), q + "w13")
                _copy(L.w2[le], need(q + "w2.weight")[:, mi0:mi0 + mi], q + "w2")
        elif phi or c.hidden_act.startswith("gelu"):
            _copy(L.w1, need(p + "mlp.fc1.weight")[I0:I0 + In], "fc1")
            if L.b1 is not None:
                _copy(L.b1, need(p + "mlp.fc1.bias")[I0:I0 + In], "fc1.bias")
            _copy(L.w2, need(p + "mlp.fc2.weight")[:, I0:I0 + In], "fc2")
            if L.b2 is not None:
                _copy(L.b2, need(p + "mlp.fc2.bias"), "fc2.bias")
        else:
            g = need(p + "mlp.gate_proj.weight")[I0:I0 + In]
            u = need(p + "mlp.up_proj.weight")[I0:I0 + In]
            _copy(L.w13, torch.cat([g, u], 0), f"{p}gate_up")
            _copy(L.w2, need(p + "mlp.down_proj.weight")[:, I0:I0 + In], f"{p}down")
    _copy(model.norm_w, need("model.final_layernorm.weight" if phi else "model.norm.weight"), "norm")
    if model.norm_b is not None:
        _copy(model.norm_b, need("model.final_layernorm.bias"), "norm.bias")
    head = get("lm_head.weight")
    if head is None or c.tie_word_embeddings:
        head = need("model.embed_tokens.weight")
    _copy(model.lm_head, head[model.vocab_start:model.vocab_end], "lm_head")
    if model.lm_head_b is not None:
        _copy(model.lm_head_b, need("lm_head.bias")[model.vocab_start:model.vocab_end], "lm_head.bias")
