"""2-SM tcgen05 GEMM (cta_group::2, CTA pairs) against an fp32 PyTorch
reference: token counts that leave ragged tiles (1, 5, 208, 300, 832),
feature counts that are not multiples of the 256-row pair tile, stream-K
tiles split over many CTA pairs (run twice: the tile counters reset
themselves), split-K, bias and a strided output."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def C():
    from swiftllm_b200.ops import cuda_ext
    return cuda_ext()


def bf(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


@pytest.mark.parametrize("T,M,K", [(1, 256, 64), (5, 640, 200), (16, 384, 4096), (208, 1000, 512),
                                   (64, 512, 4096), (256, 4096, 11008), (100, 32000, 1024),
                                   (256, 12288, 4096), (300, 4096, 1024), (832, 4096, 4096),
                                   (1000, 2048, 1000), (4096, 1536, 256)])
def test_gemm2(C, T, M, K):
    x, w, b = bf(T, K, scale=0.5), bf(M, K, scale=0.05), bf(M)
    big = torch.zeros(T, M + 64, dtype=torch.bfloat16, device="cuda")
    out = big[:, 32:32 + M]
    # automatic plan, data-parallel, and for one token tile stream-K and
    # swapped operands (tokens as the A operand)
    plans = [-1, 0] + ([1, 2] if T <= 256 else [])
    for plan in plans:
        for use_bias in (False, True):
            out.fill_(float("nan"))
            C.gemm2(out, x, w, b if use_bias else None, plan)
            r = x.float() @ w.float().t() + (b.float() if use_bias else 0)
            torch.testing.assert_close(out.float(), r, rtol=2e-2,
                                       atol=2e-2 * math.sqrt(K / 64) * 0.5, msg=f"plan {plan}")
    assert big[:, :32].abs().sum() == 0 and big[:, 32 + M:].abs().sum() == 0
    st = C.read_status(True)
    assert st[0] == 0, st


def test_gemm2_plan(C):
    bn, s, per, pairs, swap = C.gemm2_plan(12288, 832, 4096)
    assert bn == 208 and s == 1 and per == 0 and swap == 0
    # decode: tokens as A, feature tiles spread over every SM pair
    bn, s, per, pairs, swap = C.gemm2_plan(12288, 256, 4096)
    assert swap == 1 and bn % 16 == 0 and pairs * bn >= 12288 and pairs <= 74


@pytest.mark.parametrize("T,I,K", [(1, 128, 64), (37, 1376, 512), (256, 11008, 4096), (256, 2752, 4096),
                                   (300, 5504, 1024), (832, 11008, 4096)])
def test_gemm_swiglu(C, T, I, K):
    # gate/up GEMM with silu(gate) * up in the epilogue, interleaved weight
    from swiftllm_b200 import ops
    x, w13 = bf(T, K, scale=0.5), bf(2 * I, K, scale=0.05)
    out = torch.full((T, I), float("nan"), dtype=torch.bfloat16, device="cuda")
    C.gemm_swiglu(out, x, ops.interleave_gate_up(w13))
    h = x.float() @ w13.float().t()
    g, u = h[:, :I], h[:, I:]
    r = torch.nn.functional.silu(g) * u
    torch.testing.assert_close(out.float(), r, rtol=3e-2, atol=3e-2 * math.sqrt(K / 64) * 0.5)
    st = C.read_status(True)
    assert st[0] == 0, st
