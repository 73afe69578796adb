"""tiny LLaMA (2 layers, H=256, 4 q / 2 kv heads, FFN
688, V=32000, RMSNorm 1e-5, RoPE 10000, block 16), CPU fp32, random init
N(0, 0.02) seed 0; prompts of 16/32/48/64 random ids; greedy 32 tokens, EOS
ignored. Our engine (paged KV, continuous batching, C++ scheduler) must
match HF transformers' LlamaForCausalLM loaded with the same weights:
logits within fp32 tolerance and identical greedy tokens."""

import numpy as np
import pytest
import torch

from swiftllm_b200 import LLM, SamplingParams


def _hf_from_ours(model):
    from transformers import LlamaConfig, LlamaForCausalLM
    c = model.cfg
    hc = LlamaConfig(hidden_size=c.hidden_size, intermediate_size=c.intermediate_size,
                     num_hidden_layers=c.num_layers, num_attention_heads=c.num_heads,
                     num_key_value_heads=c.num_kv_heads, vocab_size=c.vocab_size,
                     rms_norm_eps=c.rms_norm_eps, rope_theta=c.rope_theta,
                     max_position_embeddings=c.max_position_embeddings,
                     tie_word_embeddings=False, attention_bias=False)
    hf = LlamaForCausalLM(hc).float().eval()
    sd = {}
    D, q, kv, I = c.head_dim, c.num_heads * c.head_dim, c.num_kv_heads * c.head_dim, c.intermediate_size
    sd["model.embed_tokens.weight"] = model.embed
    for i, L in enumerate(model.layers):
        p = f"model.layers.{i}."
        sd[p + "input_layernorm.weight"] = L.ln1
        sd[p + "self_attn.q_proj.weight"] = L.wqkv[:q]
        sd[p + "self_attn.k_proj.weight"] = L.wqkv[q:q + kv]
        sd[p + "self_attn.v_proj.weight"] = L.wqkv[q + kv:]
        sd[p + "self_attn.o_proj.weight"] = L.wo
        sd[p + "post_attention_layernorm.weight"] = L.ln2
        sd[p + "mlp.gate_proj.weight"] = L.w13[:I]
        sd[p + "mlp.up_proj.weight"] = L.w13[I:]
        sd[p + "mlp.down_proj.weight"] = L.w2
    sd["model.norm.weight"] = model.norm_w
    sd["lm_head.weight"] = model.lm_head
    missing, unexpected = hf.load_state_dict({k: v.float() for k, v in sd.items()}, strict=False)
    assert not [m for m in missing if "rotary" not in m], missing
    return hf


@pytest.fixture(scope="module")
def tiny():
    llm = LLM("tiny-llama", load_format="dummy", device="cpu", dtype="float32", max_num_seqs=8,
              seed=0)
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, 32000, size=n).tolist() for n in (16, 32, 48, 64)]
    return llm, prompts


def test_greedy_tokens_match_hf(tiny):
    llm, prompts = tiny
    outs = llm.generate(prompt_token_ids=prompts,
                        sampling_params=SamplingParams(temperature=0, max_tokens=32, ignore_eos=True),
                        use_tqdm=False)
    model = llm.llm_engine.executor.runner.model
    hf = _hf_from_ours(model)
    for p, o in zip(prompts, outs):
        with torch.no_grad():
            ids = torch.tensor([p])
            ref = hf.generate(ids, max_new_tokens=32, do_sample=False, eos_token_id=None,
                              pad_token_id=0, min_new_tokens=32)
        ref_tokens = ref[0, len(p):].tolist()
        assert o.outputs[0].token_ids == ref_tokens
        assert o.outputs[0].finish_reason.value == "length"


def test_prefill_logits_match_hf(tiny):
    llm, prompts = tiny
    model = llm.llm_engine.executor.runner.model
    hf = _hf_from_ours(model)
    from swiftllm_b200.models.decoder import AttnMeta
    p = prompts[1]
    T = len(p)
    bs = 16
    nb = (T + bs - 1) // bs
    kv = torch.zeros(nb, model.cfg.num_layers, 2, model.local_kv_heads, bs, model.cfg.head_dim)
    meta = AttnMeta(num_seqs=1, num_decode_seqs=0, num_tokens=T, max_q_len=T, max_seq_len=T,
                    positions=torch.arange(T, dtype=torch.int32),
                    slot_mapping=torch.arange(T, dtype=torch.int32),
                    q_start=torch.tensor([0, T], dtype=torch.int32),
                    seq_lens=torch.tensor([T], dtype=torch.int32),
                    block_tables=torch.arange(nb, dtype=torch.int32).view(1, nb),
                    logits_idx=torch.arange(T, dtype=torch.int32))
    with torch.no_grad():
        h = model.forward(torch.tensor(p, dtype=torch.int32), meta, kv)
        ours = model.compute_logits(h)
        ref = hf(torch.tensor([p])).logits[0].float()
    torch.testing.assert_close(ours, ref, rtol=1e-4, atol=1e-4)
