"""Counter-based random weight init (``load_format="dummy"``).

Every element of a logical (unsharded) weight gets the normal draw keyed by
(seed, tensor id) and counted by its flat index in the unsharded tensor, so
a tensor-parallel shard is exactly the matching slice of the single-rank
tensor, and the CPU and GPU generators produce the same values (up to the
last ulp of log/cos). Generator: Philox4x32-10 (Salmon et al., SC'11); normal
variates by the Box-Muller transform.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

_M0, _M1 = 0xD2511F53, 0xCD9E8D57
_W0, _W1 = 0x9E3779B9, 0xBB67AE85
_MASK = 0xFFFFFFFF


def mix_key(seed: int, tid: int) -> int:
    """64-bit Philox key for a (seed, tensor id) pair."""
    return ((seed & _MASK) << 32 | (tid & _MASK)) & 0xFFFFFFFFFFFFFFFF


def philox_torch(key: int, c0: torch.Tensor, c1: torch.Tensor):
    """Vectorised Philox4x32-10 on int64 CPU tensors holding uint32 values.
    Counter = (c0, c1, 0, 0). Returns the four output words."""
    k0, k1 = key & _MASK, (key >> 32) & _MASK
    x0, x1 = c0.clone(), c1.clone()
    x2 = torch.zeros_like(c0)
    x3 = torch.zeros_like(c0)
    for _ in range(10):
        p0 = x0 * _M0
        p1 = x2 * _M1
        hi0, lo0 = (p0 >> 32) & _MASK, p0 & _MASK
        hi1, lo1 = (p1 >> 32) & _MASK, p1 & _MASK
        x0, x1, x2, x3 = hi1 ^ x1 ^ k0, lo1, hi0 ^ x3 ^ k1, lo0
        k0 = (k0 + _W0) & _MASK
        k1 = (k1 + _W1) & _MASK
    return x0, x1, x2, x3


def normal_from_index(key: int, idx: torch.Tensor, std: float) -> torch.Tensor:
    """idx: int64 flat indices -> float32 N(0, std) draws."""
    x0, x1, _, _ = philox_torch(key, idx & _MASK, (idx >> 32) & _MASK)
    u1 = ((x0 >> 8) + 1).double() * (1.0 / 16777216.0)
    u2 = (x1 >> 8).double() * (1.0 / 16777216.0)
    z = torch.sqrt(-2.0 * torch.log(u1)) * torch.cos(2.0 * math.pi * u2)
    return (z * std).float()


def _fill_view(view: torch.Tensor, key: int, std: float, full_rows: int, full_cols: int,
               row0: int, col0: int) -> None:
    """view: [E, R, C] (or [R, C] / [C]) region of a logical [E, full_rows, full_cols]
    tensor starting at (row0, col0) in every expert slice."""
    v3 = view.reshape((-1,) + tuple(view.shape[-2:])) if view.dim() >= 2 else view.reshape(1, 1, -1)
    E, R, C = v3.shape
    if view.is_cuda:
        from ..ops import cuda_ext
        cuda_ext().init_normal(v3, key, std, full_rows, full_cols, row0, col0)
        return
    e = torch.arange(E, dtype=torch.int64).view(E, 1, 1)
    r = torch.arange(R, dtype=torch.int64).view(1, R, 1)
    c = torch.arange(C, dtype=torch.int64).view(1, 1, C)
    idx = e * (full_rows * full_cols) + (row0 + r) * full_cols + (col0 + c)
    v3.copy_(normal_from_index(key, idx.reshape(-1), std).view(E, R, C))


def fill_normal_sharded(t: torch.Tensor, spec, seed: int, tid: int, std: float) -> None:
    key = mix_key(seed, tid)
    if spec is None:
        if t.dim() == 1:
            _fill_view(t.view(1, 1, -1), key, std, 1, t.shape[0], 0, 0)
        else:
            _fill_view(t, key, std, t.shape[-2], t.shape[-1], 0, 0)
        return
    kind = spec[0]
    if kind in ("rows", "rows3"):
        full_rows, segs = spec[1], spec[2]
        if t.dim() == 1:  # bias: treat as [rows, 1]
            for lo, flo, n in segs:
                _fill_view(t[lo:lo + n].view(1, n, 1), key, std, full_rows, 1, flo, 0)
            return
        cols = t.shape[-1]
        for lo, flo, n in segs:
            _fill_view(t[..., lo:lo + n, :], key, std, full_rows, cols, flo, 0)
        return
    if kind == "exp":  # expert-parallel shard: local experts start at global e0
        e0 = spec[1]
        R, C = t.shape[-2], t.shape[-1]
        _fill_view(t, key, std, R, C, e0 * R, 0)
        return
    if kind in ("cols", "cols3"):
        full_cols, col0 = spec[1], spec[2]
        _fill_view(t, key, std, t.shape[-2], full_cols, 0, col0)
        return
    raise ValueError(kind)
