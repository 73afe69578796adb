"""Checkpoint loading: safetensors (single file and sharded index), GGUF
header/metadata/dequantisation, and conversion. Formats are the public
safetensors and GGUF layouts; the GGUF file here is written by the test."""

import json
import os
import struct

import numpy as np
import pytest
import torch

from swiftllm_b200 import LLM, SamplingParams, _core
from swiftllm_b200.loaders.convert import save_safetensors
from swiftllm_b200.models.config import load_config
from swiftllm_b200.models.decoder import DecoderModel


def _hf_state(m):
    c = m.cfg
    q, kv, I = c.q_size, c.kv_size, c.intermediate_size
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
        sd[p + "mlp.gate_proj.weight"] = L.w13[:I]
        sd[p + "mlp.up_proj.weight"] = L.w13[I:]
        sd[p + "mlp.down_proj.weight"] = L.w2
    return sd


@pytest.fixture(scope="module")
def ckpt_dir(tmp_path_factory):
    d = tmp_path_factory.mktemp("tiny_ckpt")
    cfg = load_config("tiny-llama")
    m = DecoderModel(cfg, torch.float32, "cpu")
    m.allocate()
    m.init_dummy(0)
    sd = {k: v.clone() for k, v in _hf_state(m).items()}
    keys = sorted(sd)
    half = len(keys) // 2
    save_safetensors({k: sd[k] for k in keys[:half]}, str(d / "model-00001-of-00002.safetensors"))
    save_safetensors({k: sd[k] for k in keys[half:]}, str(d / "model-00002-of-00002.safetensors"))
    idx = {"weight_map": {k: ("model-00001-of-00002.safetensors" if i < half else
                              "model-00002-of-00002.safetensors") for i, k in enumerate(keys)}}
    (d / "model.safetensors.index.json").write_text(json.dumps(idx))
    (d / "config.json").write_text(json.dumps({
        "architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 256,
        "intermediate_size": 688, "num_hidden_layers": 2, "num_attention_heads": 4,
        "num_key_value_heads": 2, "vocab_size": 32000, "rms_norm_eps": 1e-5, "rope_theta": 10000.0,
        "max_position_embeddings": 2048, "tie_word_embeddings": False}))
    return str(d)


def test_safetensors_parser(ckpt_dir):
    f = _core.SafeTensorsFile(os.path.join(ckpt_dir, "model-00001-of-00002.safetensors"))
    k = f.keys()[0]
    assert f.dtype(k) == "F32" and len(f.shape(k)) in (1, 2)
    raw = np.asarray(f.raw(k))
    assert raw.size == int(np.prod(f.shape(k))) * 4


def test_sharded_checkpoint_matches_dummy(ckpt_dir):
    sp = SamplingParams(temperature=0, max_tokens=8, ignore_eos=True)
    prompts = [[5, 6, 7, 8, 9, 10], list(range(100, 140))]
    a = LLM(ckpt_dir, device="cpu", dtype="float32", max_model_len=256).generate(
        prompt_token_ids=prompts, sampling_params=sp, use_tqdm=False)
    b = LLM("tiny-llama", load_format="dummy", device="cpu", dtype="float32",
            max_model_len=256).generate(prompt_token_ids=prompts, sampling_params=sp, use_tqdm=False)
    assert [o.outputs[0].token_ids for o in a] == [o.outputs[0].token_ids for o in b]


def test_convert_roundtrip(ckpt_dir, tmp_path):
    from swiftllm_b200.loaders.convert import convert
    out = str(tmp_path / "one.safetensors")
    n = convert(ckpt_dir, out, "bfloat16")
    f = _core.SafeTensorsFile(out)
    assert len(f.keys()) == n and f.dtype(f.keys()[0]) == "BF16"


# ---------------------------------------------------------------- GGUF
def _gguf_str(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _q8_0(x):
    x = x.reshape(-1, 32)
    d = np.abs(x).max(1) / 127.0
    d[d == 0] = 1
    q = np.round(x / d[:, None]).astype(np.int8)
    out = b"".join(np.float16(di).tobytes() + qi.tobytes() for di, qi in zip(d, q))
    return out, (q.astype(np.float32) * np.float16(d).astype(np.float32)[:, None]).reshape(-1)


def _q4_0(x):
    x = x.reshape(-1, 32)
    amax_idx = np.abs(x).argmax(1)
    mx = x[np.arange(x.shape[0]), amax_idx]
    d = mx / -8.0
    d[d == 0] = 1
    q = np.clip(np.round(x / d[:, None]) + 8, 0, 15).astype(np.uint8)
    blocks = b""
    deq = []
    for di, qi in zip(d, q):
        packed = (qi[:16] | (qi[16:] << 4)).astype(np.uint8)
        blocks += np.float16(di).tobytes() + packed.tobytes()
        deq.append((qi.astype(np.float32) - 8) * np.float32(np.float16(di)))
    return blocks, np.concatenate(deq)


def test_gguf_parse_and_dequant(tmp_path):
    rng = np.random.default_rng(0)
    a = rng.normal(size=(4, 64)).astype(np.float32)
    b = rng.normal(size=(2, 32)).astype(np.float32)
    c = rng.normal(size=(3, 32)).astype(np.float32)
    qa, ra = _q8_0(a)
    qb, rb = _q4_0(b)
    tensors = [("w.q8", a.shape, 8, qa), ("w.q4", b.shape, 2, qb), ("w.f32", c.shape, 0, c.tobytes())]
    kv = [("general.architecture", 8, _gguf_str("llama")), ("general.alignment", 4, struct.pack("<I", 32)),
          ("llama.embedding_length", 4, struct.pack("<I", 64)),
          ("tokenizer.ggml.tokens", 9, struct.pack("<IQ", 8, 2) + _gguf_str("a") + _gguf_str("b"))]
    hdr = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv))
    for k, t, v in kv:
        hdr += _gguf_str(k) + struct.pack("<I", t) + v
    off = 0
    datas = []
    for name, shape, typ, data in tensors:
        hdr += _gguf_str(name) + struct.pack("<I", len(shape))
        for dim in reversed(shape):
            hdr += struct.pack("<Q", dim)
        hdr += struct.pack("<IQ", typ, off)
        pad = (-len(data)) % 32
        datas.append(data + b"\0" * pad)
        off += len(data) + pad
    hdr += b"\0" * ((-len(hdr)) % 32)
    p = tmp_path / "t.gguf"
    p.write_bytes(hdr + b"".join(datas))
    f = _core.GgufFile(str(p))
    md = f.metadata()
    assert f.version == 3 and md["general.architecture"] == "llama"
    assert md["tokenizer.ggml.tokens"] == ["a", "b"]
    np.testing.assert_allclose(f.dequant("w.q8").reshape(-1), ra, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(f.dequant("w.q4").reshape(-1), rb, rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(f.dequant("w.f32"), c)
    assert f.dequant("w.q8").shape == (4, 64)
