"""Hot ops. CUDA tensors go to the sm_100a kernels in ``swiftllm_b200._C``;
CPU tensors go to the plain PyTorch restatements in :mod:`.reference` (the
numerics oracle and the CPU runner). A CUDA tensor never falls back: if the
extension is missing the call raises.
"""

from __future__ import annotations

import os
from typing import Optional, Tuple

import torch

from . import reference as ref

_C = None
_C_ERR: Optional[BaseException] = None
try:  # the extension is built in-tree by setup.py / __graft_entry__.build()
    from .. import _C as _C  # type: ignore
except Exception as e:  # pragma: no cover - depends on the build
    _C_ERR = e


def cuda_ext():
    """The compiled kernel module; raises loudly if it is not built."""
    if _C is None:
        raise RuntimeError(
            "swiftllm_b200._C (sm_100a kernels) is not built or failed to load: "
            f"{_C_ERR!r}. Run `python setup.py build_ext --inplace`.")
    return _C


def has_cuda_ext() -> bool:
    return _C is not None


# GEMM selection for plain bf16 projections on CUDA tensors:
#   "auto"    (default) per shape, whichever measured faster on B200: the
#             library GEMM (cuBLAS) for every plain projection except the
#             decode LM head (<= 256 tokens, >= 28k vocabulary rows), where
#             our swapped-operand tcgen05 kernel wins (58.6 vs 68.5 us at
#             256 x 32000 x 4096). Without cluster multicast (kept out of
#             all code that may run on several GPUs) our decode GEMMs re-read
#             the token tile through the L2 -> SM fabric once per feature
#             tile and lose to cuBLAS by 1.2-2x on the narrow projections.
#   "tcgen05" our kernels for every GEMM (SwiGLU fused into the gate/up
#             GEMM epilogue); tests and ablations select it.
#   "cublas"  the library GEMM everywhere (the NCCL + cuBLAS baseline arm).
# Quantized weights (FP8, int8) always run our tcgen05 kernels.
DEFAULT_GEMM_BACKEND = os.environ.get("SWIFTLLM_GEMM", "auto")
_GEMM_BACKEND = DEFAULT_GEMM_BACKEND


def set_gemm_backend(name: str) -> None:
    global _GEMM_BACKEND
    if name not in ("auto", "tcgen05", "cublas"):
        raise ValueError(name)
    _GEMM_BACKEND = name


def gemm_backend() -> str:
    return _GEMM_BACKEND


# Number of our kernels launched through this module (CUDA-graph replays add
# the count recorded at capture). Read by bench.py for "gpu_launches".
LAUNCHES = [0]


def _count(n: int = 1) -> None:
    LAUNCHES[0] += int(n)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float,
             residual: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Returns (normed, residual). With ``residual`` it is updated in place to
    residual + x first (fused add + RMSNorm)."""
    if not x.is_cuda:
        return ref.rms_norm(x, w, eps, residual)
    C = cuda_ext()
    out = torch.empty_like(x)
    if residual is None:
        C.rms_norm(out, x, w, eps)
        _count()
        return out, x
    C.fused_add_rms_norm(out, x, residual, w, eps)
    _count()
    return out, residual


def layer_norm(x, w, b, eps, residual=None):
    if not x.is_cuda:
        return ref.layer_norm(x, w, b, eps, residual)
    C = cuda_ext()
    out = torch.empty_like(x)
    if residual is None:
        C.layer_norm(out, x, w, b, eps)
        _count()
        return out, x
    C.fused_add_layer_norm(out, x, residual, w, b, eps)
    _count()
    return out, residual


class Fp8Weight:
    """A linear weight stored as E4M3 (uint8 bits) with one fp32 scale per
    output feature: w ~= q * scale[:, None]."""

    def __init__(self, q: torch.Tensor, scale: torch.Tensor):
        self.q = q
        self.scale = scale

    @property
    def shape(self):
        return self.q.shape

    @property
    def device(self):
        return self.q.device

    def dequantize(self) -> torch.Tensor:
        return self.q.view(torch.float8_e4m3fn).float() * self.scale[:, None]


class Int8Weight:
    """A linear weight stored as symmetric int8 with one fp32 scale per
    output feature (W8A8: activations are quantized per token before each
    GEMM, int32 accumulation on tcgen05 kind::i8)."""

    def __init__(self, q: torch.Tensor, scale: torch.Tensor):
        self.q = q
        self.scale = scale

    @property
    def shape(self):
        return self.q.shape

    @property
    def device(self):
        return self.q.device

    def dequantize(self) -> torch.Tensor:
        return self.q.float() * self.scale[:, None]


from . import int4  # noqa: E402
from .int4 import Int4Weight, Nvfp4Weight  # noqa: E402


def quantize_s8(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-row symmetric int8: (int8 [R, K], fp32 scale [R]), scale =
    max|row| / 127, round to nearest even."""
    x2 = x.reshape(-1, x.shape[-1])
    if not x2.is_cuda:
        s = (x2.float().abs().amax(-1) / 127.0).clamp_min(1e-12)
        q = torch.round(x2.float() / s[:, None]).clamp(-127, 127).to(torch.int8)
        return q, s
    q = torch.empty(x2.shape, dtype=torch.int8, device=x2.device)
    s = torch.empty(x2.shape[0], dtype=torch.float32, device=x2.device)
    cuda_ext().quantize_s8(q, s, x2)
    _count()
    return q, s


def int8_weight(w: torch.Tensor) -> Int8Weight:
    q, s = quantize_s8(w)
    return Int8Weight(q, s)


def _linear_int8(x, w: Int8Weight, b, out):
    xq, xs = quantize_s8(x)
    if not x.is_cuda:
        y = (xq.float() * xs[:, None]) @ w.dequantize().t()
        if b is not None:
            y = y + b.float()
        y = y.to(x.dtype).reshape(x.shape[:-1] + (w.shape[0],))
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(x.shape[:-1] + (w.shape[0],), dtype=x.dtype, device=x.device)
    _count(cuda_ext().gemm_s8(out, xq, xs, w.q, w.scale, b))
    return out


def quantize_e4m3(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-row E4M3 quantisation: (uint8 bits [R, K], fp32 scale [R]),
    scale = max|row| / 448."""
    x2 = x.reshape(-1, x.shape[-1])
    if not x2.is_cuda:
        s = (x2.float().abs().amax(-1) / 448.0).clamp_min(1e-12)
        q = (x2.float() / s[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
        return q, s
    q = torch.empty(x2.shape, dtype=torch.uint8, device=x2.device)
    s = torch.empty(x2.shape[0], dtype=torch.float32, device=x2.device)
    cuda_ext().quantize_e4m3(q, s, x2)
    _count()
    return q, s


def fp8_weight(w: torch.Tensor) -> Fp8Weight:
    q, s = quantize_e4m3(w)
    return Fp8Weight(q, s)


def _linear_fp8(x, w: Fp8Weight, b, out):
    if not x.is_cuda:
        xq, xs = quantize_e4m3(x)
        xd = xq.view(torch.float8_e4m3fn).float() * xs[:, None]
        y = xd @ w.dequantize().t()
        if b is not None:
            y = y + b.float()
        y = y.to(x.dtype).reshape(x.shape[:-1] + (w.shape[0],))
        if out is not None:
            out.copy_(y)
            return out
        return y
    xq, xs = quantize_e4m3(x)
    if out is None:
        out = torch.empty(x.shape[:-1] + (w.shape[0],), dtype=x.dtype, device=x.device)
    _count(cuda_ext().gemm_e4m3(out, xq, xs, w.q, w.scale, b))
    return out


def _library_faster(x: torch.Tensor, w: torch.Tensor) -> bool:
    """"auto" GEMM selection: True where cuBLAS measured faster (every plain
    projection but the decode LM head)."""
    return not (x.numel() // x.shape[-1] <= 256 and w.shape[0] >= 28000)


def linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None,
           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if isinstance(w, Fp8Weight):
        return _linear_fp8(x, w, b, out)
    if isinstance(w, Int8Weight):
        return _linear_int8(x, w, b, out)
    if isinstance(w, Int4Weight):
        return int4.linear(x, w, b, out)
    if isinstance(w, Nvfp4Weight):
        return int4.linear_nvfp4(x, w, b, out)
    if not x.is_cuda:
        return ref.linear(x, w, b)
    if _GEMM_BACKEND == "cublas" or (_GEMM_BACKEND == "auto" and _library_faster(x, w)):
        if w.shape[1] != x.shape[-1]:  # weight zero-padded at load
            x = torch.nn.functional.pad(x, (0, w.shape[1] - x.shape[-1]))
        if out is None:
            return torch.nn.functional.linear(x, w, b)
        x2, o2 = x.reshape(-1, x.shape[-1]), out.view(-1, out.shape[-1])
        if b is None:
            torch.matmul(x2, w.t(), out=o2)
        else:
            torch.addmm(b, x2, w.t(), out=o2)
        return out
    C = cuda_ext()
    if out is None:
        out = torch.empty(x.shape[:-1] + (w.shape[0],), dtype=x.dtype, device=x.device)
    K = x.shape[-1]
    if K % 8:
        # TMA rows must be 16-byte multiples: zero-pad K (odd shard widths,
        # e.g. a small FFN split over many ranks). Model weights arrive
        # padded already (DecoderModel.pad_k); only the activation is padded
        # per call.
        pad = 8 - K % 8
        x = torch.nn.functional.pad(x, (0, pad))
        if w.shape[1] == K:
            w = torch.nn.functional.pad(w, (0, pad))
    elif w.shape[1] != K:
        raise ValueError(f"linear: weight K {w.shape[1]} does not match input K {K}")
    _count(C.gemm(out, x, w, b))
    return out


def interleave_gate_up(w13: torch.Tensor) -> torch.Tensor:
    """[gate rows; up rows] -> rows (gate_0, up_0, gate_1, up_1, ...), the
    layout ``linear_swiglu`` reads."""
    I = w13.shape[0] // 2
    return torch.stack((w13[:I], w13[I:]), dim=1).reshape(w13.shape).contiguous()


def linear_swiglu(x: torch.Tensor, w13_il: torch.Tensor) -> torch.Tensor:
    """silu(x . gate^T) * (x . up^T) for an interleaved gate/up weight, the
    activation applied in the GEMM epilogue (one kernel, [T, I] written)."""
    if not x.is_cuda:
        g = ref.linear(x, w13_il[0::2])
        u = ref.linear(x, w13_il[1::2])
        return ref.silu_and_mul(torch.cat([g, u], dim=-1))
    out = torch.empty(x.shape[:-1] + (w13_il.shape[0] // 2,), dtype=x.dtype, device=x.device)
    _count(cuda_ext().gemm_swiglu(out, x, w13_il))
    return out


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    if not x.is_cuda:
        return ref.silu_and_mul(x)
    out = torch.empty(x.shape[:-1] + (x.shape[-1] // 2,), dtype=x.dtype, device=x.device)
    cuda_ext().silu_and_mul(out, x)
    _count()
    return out


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    if not x.is_cuda:
        return ref.gelu_tanh(x)
    out = torch.empty_like(x)
    cuda_ext().gelu_tanh(out, x)
    _count()
    return out


def embedding(ids: torch.Tensor, w: torch.Tensor, vocab_start: int = 0,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Rows of ``w`` for ``ids``; with ``vocab_start`` (vocab-parallel shard)
    ids outside [vocab_start, vocab_start + rows) give zero rows."""
    if not ids.is_cuda:
        local = ids.long() - vocab_start
        ok = (local >= 0) & (local < w.shape[0])
        res = w[local.clamp(0, w.shape[0] - 1)].clone()
        res[~ok] = 0
        if out is not None:
            out.copy_(res)
            return out
        return res
    if out is None:
        out = torch.empty((ids.shape[0], w.shape[1]), dtype=w.dtype, device=w.device)
    cuda_ext().embedding(out, ids, w, vocab_start)
    _count()
    return out


def qkv_rope_cache(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor,
                   kv_cache: torch.Tensor, layer: int, slot_mapping: torch.Tensor,
                   num_heads: int, num_kv_heads: int, head_dim: int, rotary_dim: int,
                   bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Split packed qkv [T, (Hq + 2 Hkv) D], add bias, rotate q and k (neox),
    write k and v into the paged cache at ``slot_mapping``; returns q
    [T, Hq, D]."""
    T = qkv.shape[0]
    if not qkv.is_cuda:
        if bias is not None:
            qkv = (qkv.float() + bias.float()).to(qkv.dtype)
        q = qkv[:, :num_heads * head_dim].reshape(T, num_heads, head_dim)
        k = qkv[:, num_heads * head_dim:(num_heads + num_kv_heads) * head_dim]
        k = k.reshape(T, num_kv_heads, head_dim)
        v = qkv[:, (num_heads + num_kv_heads) * head_dim:].reshape(T, num_kv_heads, head_dim)
        q = ref.apply_rope(q, positions, cos_sin, rotary_dim)
        k = ref.apply_rope(k, positions, cos_sin, rotary_dim)
        ref.write_kv(kv_cache[:, layer, 0], kv_cache[:, layer, 1], k, v, slot_mapping)
        return q
    q = torch.empty((T, num_heads, head_dim), dtype=qkv.dtype, device=qkv.device)
    cuda_ext().qkv_rope_cache(q, qkv, positions, cos_sin, kv_cache, layer, slot_mapping,
                              num_heads, num_kv_heads, head_dim, rotary_dim, bias)
    _count()
    return q


def attention(q: torch.Tensor, kv_cache: torch.Tensor, layer: int, meta,
              scale: float, sliding_window: Optional[int] = None,
              alibi_slopes: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Paged attention for a mixed batch: rows [0, num_decode) are single-token
    decode queries, the rest are (chunked) prefills reading the cached prefix.
    ``alibi_slopes`` (fp32 [num_heads]) adds slope * (key pos - query pos) to
    every score (ALiBi); those calls run the CUDA-core decode and mma.sync
    prefill kernels.
    """
    if not q.is_cuda:
        return ref.paged_attention(q, kv_cache[:, layer, 0], kv_cache[:, layer, 1],
                                   meta.block_tables, meta.q_start, meta.seq_lens, scale,
                                   sliding_window, alibi_slopes)
    C = cuda_ext()
    out = torch.empty_like(q)
    win = int(sliding_window or 0)
    nd = meta.num_decode_seqs
    if nd > 0:
        _count(C.paged_decode(out, q, kv_cache, layer, meta.block_tables, meta.seq_lens, nd,
                              meta.decode_splits, scale, win, meta.decode_workspace, alibi_slopes))
    if meta.num_seqs > nd:
        C.paged_prefill(out, q, kv_cache, layer, meta.block_tables, meta.q_start,
                        meta.seq_lens, nd, meta.num_seqs, meta.max_q_len, scale, win, -1,
                        alibi_slopes)
        _count()
    return out


def copy_blocks(kv_cache: torch.Tensor, pairs: torch.Tensor) -> None:
    """Copy whole KV blocks (all layers) src -> dst; pairs int32 [n, 2]."""
    if pairs.numel() == 0:
        return
    if not kv_cache.is_cuda:
        p = pairs.long()
        kv_cache[p[:, 1]] = kv_cache[p[:, 0]]
        return
    cuda_ext().copy_blocks(kv_cache, pairs)
    _count()
