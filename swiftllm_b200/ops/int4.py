"""Weight-only int4 (W4A16) with per-group scales and zero points: the
tile-packed layout the tcgen05 kernel reads, round-to-nearest quantisation,
and conversion of GPTQ / AWQ checkpoint tensors.

Parity: crates/swiftllm-cuda/src/bindings.rs:245-288 (gemm_int4 declared
with group scales) and crates/swiftllm-core/src/config.rs:184-215 (GPTQ /
AWQ quantisation methods); the reference ships neither a kernel nor a
checkpoint converter.

Dequantisation: w[m, k] = bf16((q[m, k] - z[g, m]) * s[g, m]), g = k // group,
q and z in [0, 15]. GPTQ and AWQ both use this form; they differ only in how
the nibbles are packed into int32 words (see ``from_gptq`` / ``from_awq``).
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

BM, BK = 128, 64

# Inside one packed 32-bit word of the kernel layout, nibble position i holds
# element _KPERM[i] of the 8-element K chunk (elements 2j at bit 4j, 2j + 1 at
# bit 16 + 4j), so one shift and mask yields a bf16 pair of neighbours.
_KPERM = (0, 2, 4, 6, 1, 3, 5, 7)
# AWQ packs column 8c + _AWQ_ORDER[i] into nibble i of word c.
_AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)


def _code_tiles(K: int) -> int:
    """64-wide code tiles along K: an even count, since the kernel's k step
    reads two consecutive tiles (128 input features)."""
    return 2 * math.ceil(K / (2 * BK))


class Int4Weight:
    """A linear weight [M, K] as int4 codes with per-(group, feature) scale
    and zero point.

    qp: uint8 [ceil(M/128), 2*ceil(K/128), 128, 32] (tile-packed codes)
    sz: int32 [G, ceil(M/128)*128], each word the bf16 pair (128 + z, s)
    """

    def __init__(self, qp: torch.Tensor, sz: torch.Tensor, M: int, K: int, group: int):
        self.qp, self.sz, self.M, self.K, self.group = qp, sz, M, K, group

    @property
    def shape(self):
        return (self.M, self.K)

    @property
    def device(self):
        return self.qp.device

    def codes(self) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(q uint8 [M, K], z float [G, M], s float [G, M]) unpacked again."""
        Mt, Kt = self.qp.shape[:2]
        b = self.qp.permute(0, 2, 1, 3).reshape(Mt * BM, Kt * 8, 4).to(torch.int32)
        nib = torch.stack([b & 15, b >> 4], -1).reshape(Mt * BM, Kt * 8, 8)  # nibble positions
        q = torch.empty_like(nib)
        # byte j holds nibble positions 2j (low) and 2j + 1 (high)
        for pos, e in enumerate(_KPERM):
            q[..., e] = nib[..., pos]
        q = q.reshape(Mt * BM, Kt * BK)[: self.M, : self.K].to(torch.uint8)
        pair = self.sz.view(torch.int16).reshape(self.sz.shape[0], -1, 2)
        G = math.ceil(self.K / self.group)
        zb = pair[:G, :, 0].view(torch.bfloat16).float()[:, : self.M]
        s = pair[:G, :, 1].view(torch.bfloat16).float()[:, : self.M]
        return q, zb - 128.0, s

    def dequantize(self) -> torch.Tensor:
        """[M, K] fp32 holding exactly the bf16 values the kernel multiplies."""
        q, z, s = self.codes()
        g = torch.arange(self.K, device=q.device) // self.group
        w = (q.float() - z[g].t()) * s[g].t()
        return w.to(torch.bfloat16).float()


def pack(q: torch.Tensor, z: torch.Tensor, s: torch.Tensor, group: int) -> Int4Weight:
    """q uint8 [M, K] codes in [0, 15], z / s [G, M] per group (G = ceil(K /
    group)), group a multiple of 64 -> Int4Weight on q's device. z may be
    any integer in [0, 16] (GPTQ v1 checkpoints reach 16)."""
    if group % BK:
        raise ValueError(f"int4 group size must be a multiple of {BK}, got {group}")
    M, K = q.shape
    Mt, Kt = math.ceil(M / BM), _code_tiles(K)
    G = math.ceil(Kt * BK / group)
    dev = q.device
    qpad = torch.zeros(Mt * BM, Kt * BK, dtype=torch.uint8, device=dev)
    qpad[:M, :K] = q
    e = qpad.view(Mt * BM, Kt * 8, 8)
    lo = e[..., list(_KPERM[0::2])]  # nibble positions 0, 2, 4, 6
    hi = e[..., list(_KPERM[1::2])]  # nibble positions 1, 3, 5, 7
    bytes_ = (lo | (hi << 4)).reshape(Mt * BM, Kt, 32)
    qp = bytes_.view(Mt, BM, Kt, 32).permute(0, 2, 1, 3).contiguous()
    zp = torch.zeros(G, Mt * BM, dtype=torch.float32, device=dev)
    sp = torch.zeros(G, Mt * BM, dtype=torch.float32, device=dev)
    zp[: z.shape[0], :M] = z.float()
    sp[: s.shape[0], :M] = s.float()
    pair = torch.stack([(zp + 128.0).to(torch.bfloat16).view(torch.int16),
                        sp.to(torch.bfloat16).view(torch.int16)], -1).contiguous()
    sz = pair.view(torch.int32).reshape(G, Mt * BM)
    return Int4Weight(qp, sz, M, K, group)


def quantize(w: torch.Tensor, group: int = 128) -> Int4Weight:
    """Per-group int4 codes for w [M, K].

    A group whose values already lie on a grid of at most 16 levels (the
    dequantised weights of a GPTQ / AWQ checkpoint) keeps that grid: the step
    s is the smallest gap between its distinct values, z = -round(min / s),
    so the checkpoint's codes come back (zero point shifted if the codes
    left levels unused; (q - z) * s is unchanged). Every other group is
    quantised asymmetrically to nearest: s = (max - min) / 15 over a range
    that includes 0, z = round(-min / s), q = clamp(round(w / s) + z, 0, 15).
    Scales are held in bf16.
    """
    M, K = w.shape
    G = math.ceil(K / group)
    wf = torch.zeros(M, G * group, dtype=torch.float32, device=w.device)
    wf[:, :K] = w.float()
    g = wf.view(M, G, group)
    # round to nearest
    lo = g.amin(-1).clamp(max=0.0)
    hi = g.amax(-1).clamp(min=0.0)
    s = ((hi - lo) / 15.0).clamp_min(1e-8)
    z = torch.round(-lo / s).clamp(0, 15)
    # grid snap (padding columns are 0, which lies on every grid through 0;
    # groups without 0 on their grid fall back to round to nearest)
    srt = g.sort(-1).values
    gap = srt.diff(dim=-1)
    tol = 1e-6 * srt.abs().amax(-1, keepdim=True).clamp_min(1e-30)
    gs = torch.where(gap > tol, gap, torch.full_like(gap, float("inf"))).amin(-1)
    gs = torch.where(torch.isfinite(gs), gs, torch.ones_like(gs))
    r = g / gs[..., None]
    rr = torch.round(r)
    on_grid = ((r - rr).abs().amax(-1) < 1e-3) & (rr.amax(-1) - rr.amin(-1) <= 15)
    s = torch.where(on_grid, gs, s)
    z = torch.where(on_grid, -rr.amin(-1), z)
    s = s.to(torch.bfloat16).float()
    q = torch.where(on_grid[..., None], rr + z[..., None],
                    torch.round(g / s[..., None]) + z[..., None]).clamp(0, 15).to(torch.uint8)
    return pack(q.view(M, G * group)[:, :K], z.t().contiguous(), s.t().contiguous(), group)


def _unpack_k(words: torch.Tensor) -> torch.Tensor:
    """int32 [R, C] -> [R * 8, C]: nibble j of word (r, c) becomes row 8r + j."""
    sh = torch.arange(0, 32, 4, device=words.device, dtype=torch.int32)
    n = (words.unsqueeze(1) >> sh.view(1, 8, 1)) & 15
    return n.reshape(words.shape[0] * 8, words.shape[1])


def _unpack_n(words: torch.Tensor, order=None) -> torch.Tensor:
    """int32 [R, C] -> [R, C * 8]: nibble i of word (r, c) becomes column
    8c + order[i] (order = identity when None)."""
    sh = torch.arange(0, 32, 4, device=words.device, dtype=torch.int32)
    n = (words.unsqueeze(-1) >> sh) & 15  # [R, C, 8] by nibble position
    if order is not None:
        out = torch.empty_like(n)
        for i, col in enumerate(order):
            out[..., col] = n[..., i]
        n = out
    return n.reshape(words.shape[0], words.shape[1] * 8)


def from_gptq(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
              g_idx: Optional[torch.Tensor] = None, zero_offset: int = 1,
              group: Optional[int] = None):
    """GPTQ tensors -> (q [N, K] uint8, z [G, N], s [G, N], group).

    qweight int32 [K/8, N]: element k = 8i + j at bits 4j of word (i, n);
    qzeros int32 [G, N/8] packed along N; scales [G, N]. The GPTQ v1
    format stores z - 1 (``zero_offset`` = 1). Only the identity group map
    (g_idx[k] == k // group, "desc_act" off) is supported. ``group``
    defaults to ceil(K / G).
    """
    q = _unpack_k(qweight.to(torch.int32)).t().contiguous()
    K = q.shape[1]
    G = scales.shape[0]
    group = group or -(-K // G)
    if g_idx is not None:
        want = torch.arange(K, device=g_idx.device) // group
        if not torch.equal(g_idx.to(torch.int64), want):
            raise NotImplementedError("GPTQ act-order (desc_act) checkpoints are not supported")
    # v1 stores (z - 1) & 15 and adds the 1 back unmasked, so a stored 15
    # means z = 16; kept as is (the kernel's zero point is any bf16 integer)
    z = (_unpack_n(qzeros.to(torch.int32)) + zero_offset).float()[:, : q.shape[0]]
    return q.to(torch.uint8), z, scales.float(), group


def from_awq(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
             group: Optional[int] = None):
    """AWQ tensors -> (q [N, K] uint8, z [G, N], s [G, N], group).

    qweight int32 [K, N/8] and qzeros int32 [G, N/8] are packed along N with
    nibble i of word c holding column 8c + (0, 2, 4, 6, 1, 3, 5, 7)[i];
    scales [G, N]; ``group`` defaults to ceil(K / G)."""
    q = _unpack_n(qweight.to(torch.int32), _AWQ_ORDER).t().contiguous()
    K = q.shape[1]
    G = scales.shape[0]
    z = _unpack_n(qzeros.to(torch.int32), _AWQ_ORDER).float()[:, : q.shape[0]]
    return q.to(torch.uint8), z, scales.float(), group or -(-K // G)


def dequantize_codes(q: torch.Tensor, z: torch.Tensor, s: torch.Tensor, group: int) -> torch.Tensor:
    """[N, K] fp32 weights (q - z) * s from unpacked codes."""
    g = torch.arange(q.shape[1], device=q.device) // group
    return (q.float() - z[g].t()) * s[g].t()


def linear(x: torch.Tensor, w: Int4Weight, b: Optional[torch.Tensor] = None,
           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x [..., K] . dequant(w)^T (+ b): the tcgen05 W4A16 kernel on CUDA,
    the dequantised fp32 maths on CPU."""
    from . import _count, cuda_ext
    if not x.is_cuda:
        y = x.float() @ w.dequantize().t()
        if b is not None:
            y = y + b.float()
        y = y.to(x.dtype).reshape(x.shape[:-1] + (w.M,))
        if out is not None:
            out.copy_(y)
            return out
        return y
    K = x.shape[-1]
    if K % 8:
        x = torch.nn.functional.pad(x, (0, 8 - K % 8))
    if out is None:
        out = torch.empty(x.shape[:-1] + (w.M,), dtype=x.dtype, device=x.device)
    _count(cuda_ext().gemm_w4a16(out, x, w.qp, w.sz, w.M, w.group, b))
    return out


# ---------------------------------------------------------------- NVFP4
# E2M1 magnitudes by 3-bit code; bit 3 of a nibble is the sign.
E2M1 = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


class Nvfp4Weight:
    """A linear weight [M, K] in NVFP4: E2M1 codes, one E4M3 scale per 16
    input features, one fp32 scale per tensor; w = bf16(e2m1 * bf16(e4m3 *
    gscale)). The kernel multiplies in bf16 on the tensor cores (the codes are
    a storage format: a quarter of the bf16 weight bytes plus 1/16 for the
    block scales).

    qp: uint8 [ceil(M/128), 2*ceil(K/128), 128, 32] (same packing as int4)
    sc: int32 [2*ceil(K/128), ceil(M/128)*128], byte b = E4M3 scale of block b
    """

    def __init__(self, qp: torch.Tensor, sc: torch.Tensor, gscale: float, M: int, K: int):
        self.qp, self.sc, self.gscale, self.M, self.K = qp, sc, float(gscale), M, K

    @property
    def shape(self):
        return (self.M, self.K)

    @property
    def device(self):
        return self.qp.device

    def block_scales(self) -> torch.Tensor:
        """[M, ceil(K/16)] fp32 effective block scales bf16(e4m3 * gscale)."""
        b = self.sc.contiguous().view(torch.uint8).reshape(self.sc.shape[0], -1, 4)  # [Kt, Mpad, 4]
        e4 = b.view(torch.float8_e4m3fn).float().permute(1, 0, 2).reshape(b.shape[1], -1)
        return (e4 * self.gscale).to(torch.bfloat16).float()[: self.M]

    def dequantize(self) -> torch.Tensor:
        """[M, K] fp32 holding exactly the bf16 values the kernel multiplies."""
        q = Int4Weight(self.qp, torch.zeros(1, self.qp.shape[0] * BM, dtype=torch.int32,
                                             device=self.qp.device), self.M, self.K, BK).codes()[0]
        lut = torch.tensor(E2M1, device=q.device)
        v = lut[(q & 7).long()] * torch.where((q & 8) > 0, -1.0, 1.0)
        s = self.block_scales()[:, torch.arange(self.K, device=q.device) // 16]
        return (v * s).to(torch.bfloat16).float()


def quantize_nvfp4(w: torch.Tensor) -> Nvfp4Weight:
    """NVFP4 quantisation of w [M, K]: gscale = amax(w) / (448 * 6); per block
    of 16 input features the E4M3 scale rounds amax(block) / 6 / gscale; each
    element takes the nearest E2M1 value of w / bf16(e4m3 * gscale) (ties to
    the smaller magnitude)."""
    M, K = w.shape
    Kt = _code_tiles(K)
    Mt = math.ceil(M / BM)
    wf = torch.zeros(M, Kt * BK, dtype=torch.float32, device=w.device)
    wf[:, :K] = w.float()
    blocks = wf.view(M, Kt * 4, 16)
    amax = blocks.abs().amax(-1)
    gscale = max(float(amax.max()) / (448.0 * 6.0), 1e-30)
    e4 = (amax / 6.0 / gscale).clamp(max=448.0).to(torch.float8_e4m3fn)
    eff = (e4.float() * gscale).to(torch.bfloat16).float()
    x = blocks / eff.clamp_min(1e-30)[..., None]
    grid = torch.tensor(E2M1, device=w.device)
    mag = (x.abs()[..., None] - grid).abs().argmin(-1)  # nearest, first on ties
    code = (mag | torch.where(x < 0, 8, 0)).to(torch.uint8).view(M, Kt * BK)
    qp = pack(code, torch.zeros(1, M), torch.zeros(1, M), BK).qp
    scb = torch.zeros(Mt * BM, Kt * 4, dtype=torch.uint8, device=w.device)
    scb[:M] = e4.view(torch.uint8)
    sc = scb.view(Mt * BM, Kt, 4).permute(1, 0, 2).contiguous().view(torch.int32).view(Kt, Mt * BM)
    return Nvfp4Weight(qp, sc, gscale, M, K)


def linear_nvfp4(x: torch.Tensor, w: Nvfp4Weight, b: Optional[torch.Tensor] = None,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x [..., K] . dequant(w)^T (+ b): the tcgen05 kernel on CUDA, the
    dequantised fp32 maths on CPU."""
    from . import _count, cuda_ext
    if not x.is_cuda:
        y = x.float() @ w.dequantize().t()
        if b is not None:
            y = y + b.float()
        y = y.to(x.dtype).reshape(x.shape[:-1] + (w.M,))
        if out is not None:
            out.copy_(y)
            return out
        return y
    K = x.shape[-1]
    if K % 8:
        x = torch.nn.functional.pad(x, (0, 8 - K % 8))
    if out is None:
        out = torch.empty(x.shape[:-1] + (w.M,), dtype=x.dtype, device=x.device)
    _count(cuda_ext().gemm_nvfp4w(out, x, w.qp, w.sc, w.M, w.gscale, b))
    return out
