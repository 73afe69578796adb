"""W4A16 int4 weights on CPU: the tile-packed layout (checked against an
emulation of the kernel's shift/mask/bf16 dequantisation), round-to-nearest
quantisation, GPTQ / AWQ unpacking, a GPTQ checkpoint loaded through the
engine, and an int4 tiny model generating."""

import json

import numpy as np
import pytest
import torch

from swiftllm_b200 import LLM, SamplingParams, ops
from swiftllm_b200.loaders.convert import save_safetensors
from swiftllm_b200.models.config import load_config
from swiftllm_b200.models.decoder import DecoderModel
from swiftllm_b200.ops import int4


def _bf16_bits_to_float(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def _kernel_emulation(W: int4.Int4Weight) -> torch.Tensor:
    """What the dequantisation warps write: for each row and 8-element chunk,
    word -> ((word >> 4j) & 0x000F000F) | 0x43004300 as a bf16 pair, minus
    (128 + z), times s (each step rounded to bf16, as the bf16x2 ops do)."""
    Mt, Kt = W.qp.shape[:2]
    words = W.qp.permute(0, 2, 1, 3).reshape(Mt * 128, Kt * 8, 4).numpy().view(np.uint32)[..., 0]
    pair = W.sz.numpy().view(np.uint16).reshape(W.sz.shape[0], -1, 2)
    zb = _bf16_bits_to_float(pair[..., 0])
    s = _bf16_bits_to_float(pair[..., 1])
    out = np.zeros((Mt * 128, Kt * 64), np.float32)
    g = (np.arange(Kt * 64) // W.group)
    for j in range(4):
        p = ((words >> (4 * j)) & 0x000F000F) | 0x43004300
        lo = _bf16_bits_to_float((p & 0xFFFF).astype(np.uint16))
        hi = _bf16_bits_to_float((p >> 16).astype(np.uint16))
        for half, v in ((0, lo), (1, hi)):
            cols = np.arange(Kt * 8) * 8 + 2 * j + half
            d = v - zb[g[cols]].T  # exact: small integers
            prod = torch.from_numpy(d * s[g[cols]].T).to(torch.bfloat16).float().numpy()
            out[:, cols] = prod
    return torch.from_numpy(out[: W.M, : W.K])


@pytest.mark.parametrize("M,K,group", [(200, 300, 128), (128, 64, 64), (300, 688, 128)])
def test_pack_layout_matches_kernel_emulation(M, K, group):
    torch.manual_seed(M + K)
    w = torch.randn(M, K) * 0.05
    W = int4.quantize(w, group)
    assert W.qp.shape == (-(-M // 128), 2 * -(-K // 128), 128, 32)
    assert torch.equal(_kernel_emulation(W), W.dequantize())
    # round to nearest: error at most half a step (plus the bf16 rounding)
    q, z, s = W.codes()
    step = s[torch.arange(K) // group].t()
    assert ((W.dequantize() - w).abs() <= 0.5 * step + 0.01 * w.abs() + 1e-6).all()


def test_pack_codes_roundtrip():
    q = torch.randint(0, 16, (130, 192), dtype=torch.uint8)
    z = torch.randint(0, 17, (3, 130)).float()
    s = torch.rand(3, 130).to(torch.bfloat16).float()
    a, b, c = int4.pack(q, z, s, 64).codes()
    assert torch.equal(a, q) and torch.equal(b, z) and torch.equal(c, s)


def _to_gptq(q, z, s, group):
    """Codes [N, K] / z, s [G, N] -> GPTQ v1 tensors (z stored minus one)."""
    N, K = q.shape
    qt = q.t().long()
    qw = torch.zeros(K // 8, N, dtype=torch.int64)
    for j in range(8):
        qw |= qt[j::8] << (4 * j)
    zs = (z.long() - 1) & 15
    qz = torch.zeros(z.shape[0], N // 8, dtype=torch.int64)
    for j in range(8):
        qz |= zs[:, j::8] << (4 * j)
    wrap = lambda t: ((t + 2 ** 31) % 2 ** 32 - 2 ** 31).to(torch.int32)  # noqa: E731
    return wrap(qw), wrap(qz), s.half()


def _to_awq(q, z, s):
    order = (0, 2, 4, 6, 1, 3, 5, 7)
    qt = q.t().long()
    qw = torch.zeros(qt.shape[0], q.shape[0] // 8, dtype=torch.int64)
    qz = torch.zeros(z.shape[0], q.shape[0] // 8, dtype=torch.int64)
    for i, col in enumerate(order):
        qw |= qt[:, col::8] << (4 * i)
        qz |= z.long()[:, col::8] << (4 * i)
    wrap = lambda t: ((t + 2 ** 31) % 2 ** 32 - 2 ** 31).to(torch.int32)  # noqa: E731
    return wrap(qw), wrap(qz), s.half()


def test_gptq_and_awq_unpack():
    N, K, g = 16, 256, 128
    q = torch.randint(0, 16, (N, K), dtype=torch.uint8)
    z = torch.randint(1, 16, (K // g, N)).float()
    s = torch.rand(K // g, N).half().float()
    Q, Z, S, G = int4.from_gptq(*_to_gptq(q, z, s, g))
    assert torch.equal(Q, q) and torch.equal(Z, z) and torch.equal(S, s) and G == g
    Q, Z, S, G = int4.from_awq(*_to_awq(q, z, s))
    assert torch.equal(Q, q) and torch.equal(Z, z) and G == g
    with pytest.raises(NotImplementedError):
        int4.from_gptq(*_to_gptq(q, z, s, g), g_idx=torch.arange(K) % 2)


def test_int4_linear_matches_dequantized():
    x, w, b = torch.randn(5, 256), torch.randn(96, 256) * 0.1, torch.randn(96)
    W = int4.quantize(w, 64)
    y = ops.linear(x, W, b)
    ref = x @ W.dequantize().t() + b
    assert torch.allclose(y, ref, atol=1e-4, rtol=1e-4)
    assert (y - (x @ w.t() + b)).abs().max() < 0.1 * ref.abs().max()


def test_int4_model_generates():
    sp = SamplingParams(temperature=0, max_tokens=12, ignore_eos=True)
    a = LLM("tiny-llama", load_format="dummy", device="cpu", dtype="float32", max_model_len=128,
            quantization="int4")
    out = a.generate(prompt_token_ids=[[5, 6, 7, 8, 9, 10, 11, 12]], sampling_params=sp,
                     use_tqdm=False)
    assert isinstance(a.llm_engine.executor.runner.model.layers[0].wqkv, ops.Int4Weight)
    assert len(out[0].outputs[0].token_ids) == 12


def test_gptq_checkpoint_loads_same_codes(tmp_path):
    """A GPTQ checkpoint made from the int4 codes of the dummy tiny model
    loads back to the same dequantised weights, and generates the same tokens as the
    dummy model quantised in place."""
    g = 128
    m = DecoderModel(load_config("tiny-llama"), torch.float32, "cpu")
    m.allocate()
    m.init_dummy(0)
    c = m.cfg
    qn, kvn, I = c.q_size, c.kv_size, c.intermediate_size
    sd = {"model.embed_tokens.weight": m.embed, "model.norm.weight": m.norm_w,
          "lm_head.weight": m.lm_head}
    want = {}
    for i, L in enumerate(m.layers):
        p = f"model.layers.{i}."
        sd[p + "input_layernorm.weight"] = L.ln1
        sd[p + "post_attention_layernorm.weight"] = L.ln2
        parts = {"self_attn.q_proj": L.wqkv[:qn], "self_attn.k_proj": L.wqkv[qn:qn + kvn],
                 "self_attn.v_proj": L.wqkv[qn + kvn:], "self_attn.o_proj": L.wo,
                 "mlp.gate_proj": L.w13[:I], "mlp.up_proj": L.w13[I:], "mlp.down_proj": L.w2}
        for name, w in parts.items():
            q, z, s = int4.quantize(w, g).codes()
            qw, qz, sc = _to_gptq(q, z, s, g)
            sd[p + name + ".qweight"], sd[p + name + ".qzeros"], sd[p + name + ".scales"] = qw, qz, sc
            sd[p + name + ".g_idx"] = (torch.arange(w.shape[1]) // g).to(torch.int32)
        want[i] = int4.quantize(L.wqkv, g).dequantize()
    save_safetensors({k: v.contiguous() for k, v in sd.items()}, str(tmp_path / "model.safetensors"))
    (tmp_path / "config.json").write_text(json.dumps({
        "architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 256,
        "intermediate_size": 688, "num_hidden_layers": 2, "num_attention_heads": 4,
        "num_key_value_heads": 2, "vocab_size": 32000, "rms_norm_eps": 1e-5, "rope_theta": 10000.0,
        "max_position_embeddings": 2048, "tie_word_embeddings": False,
        "quantization_config": {"quant_method": "gptq", "bits": 4, "group_size": g,
                                "desc_act": False, "sym": False}}))
    sp = SamplingParams(temperature=0, max_tokens=8, ignore_eos=True)
    prompts = [[5, 6, 7, 8, 9, 10], list(range(100, 140))]
    a = LLM(str(tmp_path), device="cpu", dtype="float32", max_model_len=256)
    oa = a.generate(prompt_token_ids=prompts, sampling_params=sp, use_tqdm=False)
    la = a.llm_engine.executor.runner.model.layers
    assert isinstance(la[0].wqkv, ops.Int4Weight)
    for i in want:
        # same grid: identical dequantised weights (codes may differ by a
        # zero-point shift where a group left its lowest level unused)
        assert torch.equal(la[i].wqkv.dequantize(), want[i])
    b = LLM("tiny-llama", load_format="dummy", device="cpu", dtype="float32", max_model_len=256,
            quantization="int4")
    ob = b.generate(prompt_token_ids=prompts, sampling_params=sp, use_tqdm=False)
    assert [o.outputs[0].token_ids for o in oa] == [o.outputs[0].token_ids for o in ob]


def _byte_perm(a, b, s):
    """CUDA __byte_perm: result byte n = byte (s >> 4n) & 7 of (b:a)."""
    src = (b.astype(np.uint64) << np.uint64(32)) | a.astype(np.uint64)
    out = np.zeros_like(a, dtype=np.uint64)
    for n in range(4):
        sel = (np.asarray(s, dtype=np.uint64) >> np.uint64(4 * n)) & np.uint64(7)
        out |= ((src >> (sel * np.uint64(8))) & np.uint64(0xFF)) << np.uint64(8 * n)
    return out.astype(np.uint32)


def _fp4_kernel_emulation(W) -> torch.Tensor:
    """The kernel's E2M1 decode (byte-permute tables, sign move) times the
    bf16 block scale, rounded to bf16 like the bf16x2 multiply."""
    Mt, Kt = W.qp.shape[:2]
    words = W.qp.permute(0, 2, 1, 3).reshape(Mt * 128, Kt * 8, 4).numpy().view(np.uint32)[..., 0]
    c = lambda v: np.full(words.shape, v, np.uint32)  # noqa: E731
    mag = words & np.uint32(0x77777777)
    se, so = mag & np.uint32(0xFFFF), mag >> np.uint32(16)
    hiE, loE = _byte_perm(c(0x3F3F3F00), c(0x40404040), se), _byte_perm(c(0xC0800000), c(0xC0804000), se)
    hiO, loO = _byte_perm(c(0x3F3F3F00), c(0x40404040), so), _byte_perm(c(0xC0800000), c(0xC0804000), so)
    a0, b0 = _byte_perm(loE, loO, 0x5140), _byte_perm(hiE, hiO, 0x5140)
    a1, b1 = _byte_perm(loE, loO, 0x7362), _byte_perm(hiE, hiO, 0x7362)
    o = [_byte_perm(a0, b0, 0x5140), _byte_perm(a0, b0, 0x7362),
         _byte_perm(a1, b1, 0x5140), _byte_perm(a1, b1, 0x7362)]
    scale = W.block_scales().numpy()  # [M, Kt*4]
    out = np.zeros((Mt * 128, Kt * 64), np.float32)
    for j in range(4):
        oj = o[j] | (((words >> np.uint32(4 * j)) & np.uint32(0x00080008)) << np.uint32(12))
        for half, v in ((0, _bf16_bits_to_float((oj & 0xFFFF).astype(np.uint16))),
                        (1, _bf16_bits_to_float((oj >> 16).astype(np.uint16)))):
            cols = np.arange(Kt * 8) * 8 + 2 * j + half
            sc = np.zeros((Mt * 128, cols.size), np.float32)
            sc[: W.M] = scale[:, cols // 16]
            out[:, cols] = torch.from_numpy(v * sc).to(torch.bfloat16).float().numpy()
    return torch.from_numpy(out[: W.M, : W.K])


@pytest.mark.parametrize("M,K", [(200, 300), (128, 64)])
def test_nvfp4_layout_matches_kernel_emulation(M, K):
    torch.manual_seed(M + K)
    w = torch.randn(M, K) * 0.05
    W = int4.quantize_nvfp4(w)
    assert torch.equal(_fp4_kernel_emulation(W), W.dequantize())
    # every element within half an E2M1 step (<= 1 unit of its block scale)
    s = W.block_scales()[:, torch.arange(K) // 16]
    assert ((W.dequantize() - w).abs() <= s * 1.0 + 0.01 * w.abs() + 1e-6).all()


def test_nvfp4_model_generates():
    sp = SamplingParams(temperature=0, max_tokens=6, ignore_eos=True)
    a = LLM("tiny-llama", load_format="dummy", device="cpu", dtype="float32", max_model_len=128,
            quantization="nvfp4")
    out = a.generate(prompt_token_ids=[[5, 6, 7, 8]], sampling_params=sp, use_tqdm=False)
    assert isinstance(a.llm_engine.executor.runner.model.layers[0].wqkv, ops.Nvfp4Weight)
    assert len(out[0].outputs[0].token_ids) == 6
