"""W4A16 int4 tcgen05 GEMM vs the fp32 product of the same dequantised
weights (the kernel's bf16 dequantisation is exact, so only fp32
accumulation order and the bf16 output rounding differ)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def C():
    from swiftllm_b200.ops import cuda_ext
    return cuda_ext()


# T covers one token, odd tails, the single-tile decode plan, split-K and
# several token tiles; M covers a partial feature tile; K a partial k step.
@pytest.mark.parametrize("T,M,K,group", [(1, 4096, 4096, 128), (37, 200, 328, 64),
                                         (256, 12288, 4096, 128), (5, 4096, 11008, 128),
                                         (300, 1000, 1024, 128), (1000, 512, 2048, 256),
                                         (1, 1024, 4224, 128)])  # 33 k steps over split-K
def test_gemm_w4a16(C, T, M, K, group):
    from swiftllm_b200.ops import int4
    torch.manual_seed(T + M + K)
    x = (torch.randn(T, K, device="cuda") * 0.5).to(torch.bfloat16)
    W = int4.quantize(torch.randn(M, K, device="cuda") * 0.05, group)
    out = torch.empty(T, M, dtype=torch.bfloat16, device="cuda")
    C.gemm_w4a16(out, x, W.qp, W.sz, M, group, None)
    r = x.float() @ W.dequantize().t()
    torch.testing.assert_close(out.float(), r, rtol=1e-2, atol=1e-2)
    st = C.read_status(True)
    assert st[0] == 0, st


def test_gemm_w4a16_bias_strided_and_linear(C):
    from swiftllm_b200 import ops
    from swiftllm_b200.ops import int4
    T, M, K = 64, 384, 512
    x = (torch.randn(T, K, device="cuda") * 0.5).to(torch.bfloat16)
    W = int4.quantize(torch.randn(M, K, device="cuda") * 0.05, 128)
    b = (torch.randn(M, device="cuda") * 0.1).to(torch.bfloat16)
    big = torch.zeros(T, M + 64, dtype=torch.bfloat16, device="cuda")
    out = big[:, :M]
    ops.linear(x, W, b, out=out)
    r = x.float() @ W.dequantize().t() + b.float()
    torch.testing.assert_close(out.float(), r, rtol=1e-2, atol=1e-2)
    assert big[:, M:].abs().max().item() == 0
    # the CPU path of the same weight gives the same numbers
    Wc = int4.Int4Weight(W.qp.cpu(), W.sz.cpu(), W.M, W.K, W.group)
    yc = ops.linear(x.cpu().float(), Wc, b.cpu().float())
    torch.testing.assert_close(out.float().cpu(), yc, rtol=1e-2, atol=1e-2)


def test_int4_model_gpu():
    from swiftllm_b200 import LLM, SamplingParams, ops
    sp = SamplingParams(temperature=0, max_tokens=16, ignore_eos=True)
    llm = LLM("tiny-llama", load_format="dummy", dtype="bfloat16", gpu_memory_utilization=0.3,
              max_model_len=256, quantization="int4")
    out = llm.generate(prompt_token_ids=[list(range(100, 164)), [7, 8, 9]], sampling_params=sp,
                       use_tqdm=False)
    assert all(len(o.outputs[0].token_ids) == 16 for o in out)
    assert isinstance(llm.llm_engine.executor.runner.model.layers[0].wqkv, ops.Int4Weight)
    st = ops.cuda_ext().read_status(True)
    assert st[0] == 0, st
    llm.shutdown()


@pytest.mark.parametrize("T,M,K", [(1, 4096, 4096), (37, 200, 328), (300, 1000, 1024),
                                   (5, 4096, 11008)])
def test_gemm_nvfp4w(C, T, M, K):
    # NVFP4 weights (E2M1 codes, E4M3 block scales, per-tensor scale) expanded
    # to bf16 in shared memory: against the fp32 product of the same weights
    from swiftllm_b200.ops import int4
    torch.manual_seed(T + M)
    x = (torch.randn(T, K, device="cuda") * 0.5).to(torch.bfloat16)
    W = int4.quantize_nvfp4(torch.randn(M, K, device="cuda") * 0.05)
    out = torch.empty(T, M, dtype=torch.bfloat16, device="cuda")
    C.gemm_nvfp4w(out, x, W.qp, W.sc, M, W.gscale, None)
    r = x.float() @ W.dequantize().t()
    torch.testing.assert_close(out.float(), r, rtol=1e-2, atol=1e-2)
    st = C.read_status(True)
    assert st[0] == 0, st


def test_nvfp4_model_gpu():
    from swiftllm_b200 import LLM, SamplingParams, ops
    sp = SamplingParams(temperature=0, max_tokens=8, ignore_eos=True)
    llm = LLM("tiny-llama", load_format="dummy", dtype="bfloat16", gpu_memory_utilization=0.3,
              max_model_len=256, quantization="nvfp4")
    out = llm.generate(prompt_token_ids=[list(range(100, 140))], sampling_params=sp, use_tqdm=False)
    assert len(out[0].outputs[0].token_ids) == 8
    assert isinstance(llm.llm_engine.executor.runner.model.layers[0].wqkv, ops.Nvfp4Weight)
    llm.shutdown()
