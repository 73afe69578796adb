"""Plain PyTorch (fp32-capable) restatements of every hot op.

These are the numerics oracles for the CUDA kernels (tests compare the
kernels against them) and the implementation of the CPU runner that checks
the tiny LLaMA configuration against HF ``transformers``. They are never
called on CUDA tensors by the engine.

Parity of the maths with the reference's declared ops:
  RMSNorm      crates/swiftllm-models/src/layers/normalization.rs:185-200
  LayerNorm    normalization.rs:203-230
  RoPE         crates/swiftllm-models/src/layers/attention.rs:216-295 (neox
               rotate_half form)
  SwiGLU       crates/swiftllm-cuda/src/bindings.rs:183-199 (silu_and_mul)
  KV write     crates/swiftllm-cuda/kernels/paged_attention.cu:167-199
               (slot -> block, offset)
  attention    paged_attention.cu:35-137 (intended maths: softmax(q.k*scale).v)
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float,
             residual: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Returns (normed, new_residual). With ``residual`` the input is first
    added to it (fused add + RMSNorm); otherwise the residual is ``x``."""
    if residual is not None:
        x = (x.float() + residual.float()).to(x.dtype)
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    return y.to(x.dtype), x


def layer_norm(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor], eps: float,
               residual: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    if residual is not None:
        x = (x.float() + residual.float()).to(x.dtype)
    y = F.layer_norm(x.float(), (x.shape[-1],), w.float(),
                     None if b is None else b.float(), eps)
    return y.to(x.dtype), x


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    d = x.shape[-1] // 2
    return (F.silu(x[..., :d].float()) * x[..., d:].float()).to(x.dtype)


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return F.gelu(x.float(), approximate="tanh").to(x.dtype)


def linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None) -> torch.Tensor:
    y = x.float() @ w.float().t()
    if b is not None:
        y = y + b.float()
    return y.to(x.dtype)


def apply_rope(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor,
               rotary_dim: int) -> torch.Tensor:
    """x: [T, H, D]; cos_sin: [max_pos, rotary_dim] (cos | sin halves).
    Neox (rotate-half) pairing over the first ``rotary_dim`` channels."""
    half = rotary_dim // 2
    cs = cos_sin[positions.long()].float()
    cos = cs[:, :half].unsqueeze(1)
    sin = cs[:, half:].unsqueeze(1)
    xf = x.float()
    x1 = xf[..., :half]
    x2 = xf[..., half:rotary_dim]
    out = xf.clone()
    out[..., :half] = x1 * cos - x2 * sin
    out[..., half:rotary_dim] = x2 * cos + x1 * sin
    return out.to(x.dtype)


def write_kv(kv_layer_k: torch.Tensor, kv_layer_v: torch.Tensor, k: torch.Tensor,
             v: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """kv_layer_*: [num_blocks, kvh, bs, D]; k, v: [T, kvh, D]."""
    bs = kv_layer_k.shape[2]
    slots = slot_mapping.long()
    valid = slots >= 0
    slots = slots[valid]
    blk, off = slots // bs, slots % bs
    kv_layer_k[blk, :, off] = k[valid].to(kv_layer_k.dtype)
    kv_layer_v[blk, :, off] = v[valid].to(kv_layer_v.dtype)


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    block_tables: torch.Tensor, q_start: torch.Tensor, seq_lens: torch.Tensor,
                    scale: float, sliding_window: Optional[int] = None,
                    alibi_slopes: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Varlen causal attention of new query tokens against the paged cache
    (which already holds these tokens). q: [T, Hq, D]; k/v_cache:
    [num_blocks, kvh, bs, D]; block_tables [S, max_blocks]; q_start [S+1];
    seq_lens [S] = cached + new tokens. Query i of a sequence sits at
    position seq_len - q_len + i."""
    T, Hq, D = q.shape
    kvh, bs = k_cache.shape[1], k_cache.shape[2]
    group = Hq // kvh
    out = torch.empty_like(q)
    qs = q_start.tolist()
    sl = seq_lens.tolist()
    for s in range(len(sl)):
        a, b = qs[s], qs[s + 1]
        if b == a:
            continue
        L = sl[s]
        nb = (L + bs - 1) // bs
        blocks = block_tables[s, :nb].long()
        k = k_cache[blocks].permute(1, 0, 2, 3).reshape(kvh, nb * bs, D)[:, :L].float()
        v = v_cache[blocks].permute(1, 0, 2, 3).reshape(kvh, nb * bs, D)[:, :L].float()
        k = k.repeat_interleave(group, 0)
        v = v.repeat_interleave(group, 0)
        qq = q[a:b].float().transpose(0, 1)  # [Hq, n, D]
        n = b - a
        scores = torch.einsum("hnd,hld->hnl", qq, k) * scale
        qpos = torch.arange(L - n, L).unsqueeze(1)
        kpos = torch.arange(L).unsqueeze(0)
        mask = kpos > qpos
        if sliding_window is not None and sliding_window > 0:
            mask = mask | (kpos <= qpos - sliding_window)
        if alibi_slopes is not None:
            scores = scores + alibi_slopes.float().view(-1, 1, 1) * (kpos - qpos).float()
        scores = scores.masked_fill(mask, float("-inf"))
        p = torch.softmax(scores, dim=-1)
        out[a:b] = torch.einsum("hnl,hld->hnd", p, v).transpose(0, 1).to(q.dtype)
    return out


def alibi_slopes(num_heads: int) -> torch.Tensor:
    """ALiBi head slopes (Press et al. 2022): geometric sequence starting at
    2^(-8/n) for the nearest power of two n, interleaving extra heads.
    Parity: crates/swiftllm-core/src/memory/paged_attention.rs:111-135."""
    n = 2 ** math.floor(math.log2(num_heads))
    base = 2.0 ** (-8.0 / n)
    slopes = [base ** (i + 1) for i in range(n)]
    if n < num_heads:
        extra_base = 2.0 ** (-4.0 / n)
        slopes += [extra_base ** (2 * i + 1) for i in range(num_heads - n)]
    return torch.tensor(slopes, dtype=torch.float32)


def moe_topk_softmax(router_logits: torch.Tensor, k: int,
                     renormalize: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
    """Mixtral routing: softmax over experts, top-k, renormalise the k weights."""
    p = torch.softmax(router_logits.float(), dim=-1)
    w, idx = torch.topk(p, k, dim=-1)
    if renormalize:
        w = w / w.sum(-1, keepdim=True)
    return w, idx.to(torch.int32)


def moe_experts(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, topk_w: torch.Tensor,
                topk_idx: torch.Tensor) -> torch.Tensor:
    """x [T, H]; w13 [E, 2I, H]; w2 [E, H, I]."""
    out = torch.zeros(x.shape, dtype=torch.float32, device=x.device)
    E = w13.shape[0]
    for e in range(E):
        rows, slot = (topk_idx == e).nonzero(as_tuple=True)
        if rows.numel() == 0:
            continue
        h = linear(x[rows], w13[e])
        h = silu_and_mul(h)
        y = linear(h, w2[e]).float()
        out.index_add_(0, rows, y * topk_w[rows, slot].unsqueeze(1).float())
    return out.to(x.dtype)
