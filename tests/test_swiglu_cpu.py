"""The interleaved gate/up layout that the fused SwiGLU GEMM reads: on CPU
``linear_swiglu`` of the interleaved weight equals the unfused path."""

import torch

from swiftllm_b200 import ops


def test_linear_swiglu_matches_unfused_cpu():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(5, 64, generator=g)
    w13 = torch.randn(2 * 48, 64, generator=g) * 0.1
    ref = ops.silu_and_mul(ops.linear(x, w13))
    got = ops.linear_swiglu(x, ops.interleave_gate_up(w13))
    torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-5)
    il = ops.interleave_gate_up(w13)
    assert torch.equal(il[0::2], w13[:48]) and torch.equal(il[1::2], w13[48:])
