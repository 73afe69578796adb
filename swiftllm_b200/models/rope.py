"""Rotary position embedding tables, with the scaling variants.

Parity: crates/swiftllm-models/src/layers/attention.rs:216-353
(RotaryEmbedding: inv_freq = base^(-2i/d), cos/sin cache; YaRNScaling) and
crates/swiftllm-core/src/config.rs:218-242 (Linear / Dynamic / YaRN /
LongRoPE). The table is [max_pos, rotary_dim] float32 holding cos in the
first half and sin in the second, consumed by the fused QKV/RoPE/KV-write
kernel. Scaling formulas follow the published methods: position
interpolation (Chen et al. 2023) for "linear", NTK-aware base scaling for
"dynamic" (applied statically at the model's maximum length), YaRN (Peng et
al. 2023) and the Llama 3.1 frequency-band rule for "llama3".
"""

from __future__ import annotations

import math
from typing import Any, Dict, Optional, Tuple

import torch


def _yarn_find_correction_dim(num_rot, dim, base, max_pos):
    return (dim * math.log(max_pos / (num_rot * 2 * math.pi))) / (2 * math.log(base))


def inv_freq_and_mscale(rotary_dim: int, base: float, scaling: Optional[Dict[str, Any]],
                        max_pos: int) -> Tuple[torch.Tensor, float, float]:
    """Returns (inv_freq [rotary_dim/2], position scale, attention mscale)."""
    idx = torch.arange(0, rotary_dim, 2, dtype=torch.float64) / rotary_dim
    inv = 1.0 / (base ** idx)
    if not scaling:
        return inv.float(), 1.0, 1.0
    kind = (scaling.get("rope_type") or scaling.get("type") or "").lower()
    factor = float(scaling.get("factor", 1.0))
    if kind == "linear":
        return inv.float(), 1.0 / factor, 1.0
    if kind == "dynamic":
        orig = int(scaling.get("original_max_position_embeddings", max_pos))
        seq = max(max_pos, orig)
        new_base = base * ((factor * seq / orig) - (factor - 1)) ** (rotary_dim / (rotary_dim - 2))
        return (1.0 / (new_base ** idx)).float(), 1.0, 1.0
    if kind == "yarn":
        orig = int(scaling.get("original_max_position_embeddings", max_pos))
        beta_fast = float(scaling.get("beta_fast", 32))
        beta_slow = float(scaling.get("beta_slow", 1))
        low = max(math.floor(_yarn_find_correction_dim(beta_fast, rotary_dim, base, orig)), 0)
        high = min(math.ceil(_yarn_find_correction_dim(beta_slow, rotary_dim, base, orig)),
                   rotary_dim - 1)
        if low == high:
            high += 0.001
        ramp = ((torch.arange(rotary_dim // 2, dtype=torch.float64) - low) / (high - low)).clamp(0, 1)
        extrap_weight = 1.0 - ramp
        inv_interp = inv / factor
        inv = inv_interp * (1 - extrap_weight) + inv * extrap_weight
        mscale = float(scaling.get("mscale", 1.0)) if "mscale" in scaling else 1.0
        attn_factor = 0.1 * math.log(factor) + 1.0 if factor > 1 else 1.0
        return inv.float(), 1.0, attn_factor * mscale
    if kind == "llama3":
        low_ff = float(scaling.get("low_freq_factor", 1.0))
        high_ff = float(scaling.get("high_freq_factor", 4.0))
        orig = int(scaling.get("original_max_position_embeddings", 8192))
        low_wl = orig / low_ff
        high_wl = orig / high_ff
        wl = 2 * math.pi / inv
        out = torch.where(wl > low_wl, inv / factor, inv)
        smooth = (orig / wl - low_ff) / (high_ff - low_ff)
        mid = (1 - smooth) * inv / factor + smooth * inv
        is_mid = (wl <= low_wl) & (wl >= high_wl)
        out = torch.where(is_mid, mid, out)
        return out.float(), 1.0, 1.0
    if kind in ("default", ""):
        return inv.float(), 1.0, 1.0
    raise ValueError(f"unsupported rope scaling type {kind!r}")


def cos_sin_table(rotary_dim: int, base: float, max_pos: int,
                  scaling: Optional[Dict[str, Any]] = None,
                  device=None) -> torch.Tensor:
    inv, pos_scale, mscale = inv_freq_and_mscale(rotary_dim, base, scaling, max_pos)
    t = torch.arange(max_pos, dtype=torch.float32) * pos_scale
    freqs = torch.outer(t, inv)
    table = torch.cat([freqs.cos() * mscale, freqs.sin() * mscale], dim=-1)
    return table.to(device=device, dtype=torch.float32).contiguous()
