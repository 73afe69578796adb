"""Mixtral-architecture MoE on the CPU runner against HF transformers'
MixtralForCausalLM with the same weights (router softmax -> top-2 ->
renormalise -> SwiGLU experts -> weighted sum)."""

import torch

from swiftllm_b200.models.config import load_config
from swiftllm_b200.models.decoder import AttnMeta, DecoderModel


def _meta(T):
    nb = (T + 15) // 16
    return AttnMeta(num_seqs=1, num_decode_seqs=0, num_tokens=T, max_q_len=T, max_seq_len=T,
                    positions=torch.arange(T, dtype=torch.int32),
                    slot_mapping=torch.arange(T, dtype=torch.int32),
                    q_start=torch.tensor([0, T], dtype=torch.int32),
                    seq_lens=torch.tensor([T], dtype=torch.int32),
                    block_tables=torch.arange(nb, dtype=torch.int32).view(1, nb),
                    logits_idx=torch.arange(T, dtype=torch.int32))


def test_tiny_mixtral_matches_hf():
    from transformers import MixtralConfig, MixtralForCausalLM
    cfg = load_config("tiny-mixtral")
    m = DecoderModel(cfg, torch.float32, "cpu")
    m.allocate()
    m.init_dummy(0)
    hc = MixtralConfig(hidden_size=cfg.hidden_size, intermediate_size=cfg.intermediate_size,
                       num_hidden_layers=cfg.num_layers, num_attention_heads=cfg.num_heads,
                       num_key_value_heads=cfg.num_kv_heads, vocab_size=cfg.vocab_size,
                       num_local_experts=cfg.num_experts, num_experts_per_tok=cfg.num_experts_per_tok,
                       rms_norm_eps=cfg.rms_norm_eps, rope_theta=cfg.rope_theta,
                       max_position_embeddings=cfg.max_position_embeddings, sliding_window=None,
                       tie_word_embeddings=False)
    hf = MixtralForCausalLM(hc).float().eval()
    q, kv = cfg.q_size, cfg.kv_size
    sd = {"model.embed_tokens.weight": m.embed, "model.norm.weight": m.norm_w,
          "lm_head.weight": m.lm_head}
    for i, L in enumerate(m.layers):
        p = f"model.layers.{i}."
        sd[p + "input_layernorm.weight"] = L.ln1
        sd[p + "post_attention_layernorm.weight"] = L.ln2
        sd[p + "self_attn.q_proj.weight"] = L.wqkv[:q]
        sd[p + "self_attn.k_proj.weight"] = L.wqkv[q:q + kv]
        sd[p + "self_attn.v_proj.weight"] = L.wqkv[q + kv:]
        sd[p + "self_attn.o_proj.weight"] = L.wo
        sd[p + "mlp.gate.weight"] = L.router
        sd[p + "mlp.experts.gate_up_proj"] = L.w13
        sd[p + "mlp.experts.down_proj"] = L.w2
    missing, _ = hf.load_state_dict(sd, strict=False)
    assert not [k for k in missing if "rotary" not in k], missing
    T = 29
    ids = torch.randint(0, cfg.vocab_size, (T,), dtype=torch.int32, generator=torch.Generator().manual_seed(3))
    kvc = torch.zeros((T + 15) // 16, cfg.num_layers, 2, cfg.num_kv_heads, 16, cfg.head_dim)
    with torch.no_grad():
        ours = m.compute_logits(m.forward(ids, _meta(T), kvc))
        ref = hf(ids.long().view(1, -1)).logits[0].float()
    torch.testing.assert_close(ours, ref, rtol=1e-4, atol=1e-4)
