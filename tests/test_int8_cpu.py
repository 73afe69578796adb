"""W8A8 int8 quantisation on CPU: the per-row quantiser, the int8 linear
against the dequantised maths, and a quantised tiny model through the
engine."""

import torch

from swiftllm_b200 import LLM, SamplingParams, ops


def test_quantize_s8_roundtrip():
    x = torch.randn(7, 256) * torch.linspace(0.1, 10, 7)[:, None]
    q, s = ops.quantize_s8(x)
    assert q.dtype == torch.int8 and s.shape == (7,) and q.abs().max() <= 127
    xd = q.float() * s[:, None]
    assert ((xd - x).abs() <= s[:, None] * 0.5 + 1e-6).all()


def test_int8_linear_matches_dequantized():
    x, w, b = torch.randn(5, 64), torch.randn(32, 64) * 0.1, torch.randn(32)
    y = ops.linear(x, ops.int8_weight(w), b)
    ref = x @ w.t() + b
    assert (y - ref).abs().max() < 0.05 * ref.abs().max()


def test_int8_model_generates():
    sp = SamplingParams(temperature=0, max_tokens=12, ignore_eos=True)
    a = LLM("tiny-llama", load_format="dummy", device="cpu", dtype="float32", max_model_len=128,
            quantization="int8")
    out = a.generate(prompt_token_ids=[[5, 6, 7, 8, 9, 10, 11, 12]], sampling_params=sp,
                     use_tqdm=False)
    assert isinstance(a.llm_engine.executor.runner.model.layers[0].wqkv, ops.Int8Weight)
    assert len(out[0].outputs[0].token_ids) == 12
