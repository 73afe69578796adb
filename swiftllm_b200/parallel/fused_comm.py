"""Fused tensor-parallel reduction over NVLink peer memory (the product
backend; NCCL is the baseline).

The row-parallel GEMMs (o_proj, down_proj) write their partial sums straight
into this rank's slot of a symmetric allocation (``reduce_buffer``); the
reduction kernel (csrc/kernels/tp_allreduce.cu) then sums all ranks'
partials with peer loads and per-block release/acquire flags, so no NCCL
call sits on the per-layer path. The vocab-parallel logits gather stays on
NCCL (one small call per step).

Fused GEMM -> all-reduce (``linear_reduce`` for o_proj and down_proj, the
default; SWIFTLLM_FUSED_GEMM_RS=0 turns it off): the GEMM epilogue stores each output row
straight into the receive buffer of the rank that owns that token
(reduce-scatter by NVLink stores, overlapped with the remaining GEMM tiles)
and publishes a completion epoch; ``tp_rs_finish`` then sums each rank's own
tokens and pushes them to every rank (all-gather by stores). Otherwise the
GEMM writes this rank's partial into its symmetric slot and ``reduce`` runs
the two-shot reduction kernel.

Layout of the symmetric allocation (bytes):
  [flags 64 KiB | in A | in B | red A | red B], each buffer (max_tokens + 8) x H
  bf16. Flags: [phase][block][rank] u32 barrier slots at 0, the fused GEMM's
  per-source completion epochs at 8 KiB. `in` doubles as the fused receive
  buffer [src rank][ceil(max_tokens / k)][H].
"""

from __future__ import annotations

import os
from typing import Optional

import torch

from ..utils.logging import get_logger
from .comm import NcclTP
from .failures import CommTimeoutError

log = get_logger(__name__)

_FLAGS_BYTES = 64 << 10
_GEMM_FLAG_OFF = 8 << 10
FUSED_GEMM = os.environ.get("SWIFTLLM_FUSED_GEMM_RS", "1") == "1"
# residual add + RMSNorm folded into the reduce's finish kernel
FUSED_NORM = os.environ.get("SWIFTLLM_FUSED_NORM", "0") == "1"
TIMEOUT_S = float(os.environ.get("SWIFTLLM_COMM_TIMEOUT", "5.0"))


class FusedTP(NcclTP):
    def __init__(self, rank: int, size: int, device: torch.device, model_cfg,
                 max_tokens: int = 8192):
        super().__init__(rank, size)
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        from ..ops import cuda_ext
        self.C = cuda_ext()
        self.device = device
        H = model_cfg.hidden_size
        self.H = H
        self.max_tokens = max_tokens
        self.max_elems = max_tokens * H
        self.s_max = (max_tokens + size - 1) // size
        self.buf_bytes = ((max_tokens + 8) * H * 2 + 255) // 256 * 256
        total = _FLAGS_BYTES + 6 * self.buf_bytes
        self.symm = symm_mem.empty(total // 2, dtype=torch.bfloat16, device=device)
        self.symm.zero_()
        torch.cuda.synchronize(device)
        self.hdl = symm_mem.rendezvous(self.symm, dist.group.WORLD)
        self.bases = [int(p) for p in self.hdl.buffer_ptrs]
        assert len(self.bases) == size
        self.epochs = torch.zeros(64, dtype=torch.int32, device=device)
        self.gemm_ctr = torch.zeros(4, dtype=torch.int32, device=device)
        self.gemm_epochs = torch.zeros(64, dtype=torch.int32, device=device)
        self.call = 0
        dist.barrier()
        log.info("fused TP comm ready: rank %d/%d, %.1f MiB symmetric", rank, size,
                 total / 2**20)

    def _off(self, kind: str, parity: int) -> int:
        base = _FLAGS_BYTES + {"in": 0, "red": 2, "res": 4}[kind] * self.buf_bytes
        return base + parity * self.buf_bytes

    def reduce_buffer(self, T: int, H: int) -> Optional[torch.Tensor]:
        """This rank's input slot for the next reduce: the producing GEMM
        stores its partial output here."""
        n = T * H
        if n > self.max_elems:
            return None
        off = self._off("in", self.call % 2) // 2
        return self.symm[off:off + n].view(T, H)

    def reduce(self, x: torch.Tensor) -> torch.Tensor:
        n = x.numel()
        if n > self.max_elems or n % 8:
            return super().reduce(x)
        parity = self.call % 2
        slot = self.reduce_buffer(x.shape[0], n // x.shape[0])
        if x.data_ptr() != slot.data_ptr():
            slot.copy_(x.view_as(slot))
        out = torch.empty_like(x)
        self.C.tp_allreduce(out, self.bases, self.rank, self._off("in", parity),
                            self._off("red", parity), self.epochs, TIMEOUT_S)
        from .. import ops
        ops._count()
        self.call += 1
        return out

    def linear_reduce(self, x: torch.Tensor, w: torch.Tensor,
                      b: Optional[torch.Tensor] = None, fused: Optional[bool] = None) -> torch.Tensor:
        """Row-parallel linear + sum over ranks: either one fused GEMM ->
        reduce-scatter kernel plus one reduce + all-gather kernel, or the GEMM
        into this rank's slot plus the two-shot reduction."""
        from .. import ops
        T, H = x.shape[0], w.shape[0]
        if self.rank != 0:
            b = None
        fused = FUSED_GEMM if fused is None else fused
        if (not fused or not isinstance(w, torch.Tensor) or x.shape[-1] % 8 or T == 0
                or T > self.max_tokens or H != self.H
                or ops.gemm_backend() != "tcgen05"):
            return self.reduce(ops.linear(x, w, b, out=self.reduce_buffer(T, H)))
        parity = self.call % 2
        in_off, red_off = self._off("in", parity), self._off("red", parity)
        n = self.C.gemm_rs(x, w, b, self.bases, self.rank, in_off, self.s_max, _GEMM_FLAG_OFF,
                           self.gemm_ctr)
        self.C.tp_rs_finish(self.bases, self.rank, in_off, red_off, self.s_max, T, H,
                            _GEMM_FLAG_OFF, self.gemm_epochs, self.epochs, TIMEOUT_S)
        ops._count(n + 1)
        self.call += 1
        return self.symm[red_off // 2:red_off // 2 + T * H].view(T, H)

    def linear_reduce_norm(self, x: torch.Tensor, w: torch.Tensor, norm_w: torch.Tensor,
                           eps: float, residual: torch.Tensor):
        """Row-parallel linear, cross-rank sum, residual add and RMSNorm:
        returns (normed, new residual) like ``ops.rms_norm(out, norm_w, eps,
        residual)``. Fused path: the GEMM -> reduce-scatter kernel, then one
        kernel that reduces each rank's own tokens, adds the residual,
        normalises and all-gathers both rows."""
        from .. import ops
        T, H = x.shape[0], w.shape[0]
        if (not (FUSED_GEMM and FUSED_NORM) or not isinstance(w, torch.Tensor) or x.shape[-1] % 8
                or T == 0 or T > self.max_tokens or H != self.H or ops.gemm_backend() != "tcgen05"
                or not residual.is_contiguous()):
            return ops.rms_norm(self.linear_reduce(x, w), norm_w, eps, residual)
        parity = self.call % 2
        in_off, out_off, res_off = (self._off("in", parity), self._off("red", parity),
                                    self._off("res", parity))
        n = self.C.gemm_rs(x, w, None, self.bases, self.rank, in_off, self.s_max, _GEMM_FLAG_OFF,
                           self.gemm_ctr)
        self.C.tp_rs_finish_norm(self.bases, self.rank, in_off, out_off, res_off, residual, norm_w,
                                 float(eps), self.s_max, T, H, _GEMM_FLAG_OFF, self.gemm_epochs,
                                 self.epochs, TIMEOUT_S)
        ops._count(n + 1)
        self.call += 1
        normed = self.symm[out_off // 2:out_off // 2 + T * H].view(T, H)
        res = self.symm[res_off // 2:res_off // 2 + T * H].view(T, H)
        return normed, res

    def close(self) -> None:
        """Release the symmetric allocation and its rendezvous handle (every
        rank calls this between steps, then a barrier, before the process
        group is destroyed)."""
        if getattr(self, "symm", None) is None:
            return
        torch.cuda.synchronize(self.device)
        self.hdl = None
        self.bases = []
        self.symm = None
        self.epochs = self.gemm_ctr = self.gemm_epochs = None

    def check(self) -> None:
        st = self.C.read_status(True)
        if st[0] == 2:
            raise CommTimeoutError(f"peer did not arrive within {TIMEOUT_S}s (site {st[1]})")
