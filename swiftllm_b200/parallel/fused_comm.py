"""Fused tensor-parallel communication over NVLink / NVSwitch (the product
backend; NCCL is the baseline).

Sequence-parallel layout of the decoder under this backend: the residual
stream is sharded by token rows (rank j keeps rows [T*j/k, T*(j+1)/k)); the
normalised activations that feed the next column-parallel GEMM are
replicated. Each row-parallel GEMM (o_proj, down_proj, the MoE combine)
stores its partial sum locally into this rank's ``in`` buffer of one
symmetric allocation; then ONE kernel (csrc/kernels/tp_nvls.cu,
``tp_reduce_norm``) per reduction

  * reduce-scatters: each rank sums the k partials of its own token rows
    with NVSwitch ``multimem.ld_reduce`` (fp32 accumulation in the switch)
    or, without a multicast object, k NVLink peer loads;
  * adds its residual shard and applies the next sub-block's RMSNorm;
  * all-gathers: stores the normalised rows into every rank's ``out``
    buffer with one ``multimem.st`` (or k peer stores).

The next QKV / gate_up GEMM then reads ``out`` locally. Vocab-parallel
greedy sampling (``vocab_greedy``) exchanges one (max, argmax, sum-exp)
candidate per row and rank instead of gathering fp32 logits.

Layout of the symmetric allocation (bytes):
  [counters 36 KiB | in | out | out2 | cand | gather]
  counters: reduce_norm blocks at 0, plain all-reduce blocks at 1 KiB,
  vocab rows at 4 KiB (up to 7168 rows), logits-gather blocks at 32 KiB;
  in / out / out2: (max_tokens + 8) x H bf16; cand: k x max_rows float4;
  gather: 512 x V fp32 (full-vocabulary logits of sampled / logprob steps,
  ``gather_vocab``).
``SWIFTLLM_MULTIMEM=0`` forces the peer-load path (no multicast object).

Parity: crates/swiftllm-core/src/execution/tensor_parallel.rs (all_reduce /
all_gather / reduce_scatter :115-141, CommunicationBackend :55-63) and
crates/swiftllm-models/src/layers/mod.rs (ColumnParallelLinear gather
:113-118, RowParallelLinear reduce :145-149).
"""

from __future__ import annotations

import os
from typing import Optional, Tuple

import torch

from ..utils.logging import get_logger
from .comm import NcclTP
from .failures import CommTimeoutError

log = get_logger(__name__)

_CTR_BYTES = 36 << 10
_CTR_NORM, _CTR_AR, _CTR_VOCAB, _CTR_GATHER = 0, 1 << 10, 4 << 10, 32 << 10
_GA_BLOCKS = 64           # kGaBlocks in tp_nvls.cu
_GATHER_ROWS = 512        # sampled rows the fused logits gather holds (more: NCCL)
_RN_BLOCKS = 128          # kRnBlocks in tp_nvls.cu
_MAX_ROWS = 7168          # vocab counters fit the counter region
TIMEOUT_S = float(os.environ.get("SWIFTLLM_COMM_TIMEOUT", "5.0"))
USE_MULTIMEM = os.environ.get("SWIFTLLM_MULTIMEM", "1") != "0"


class FusedTP(NcclTP):
    sequence_parallel = True

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
        self.max_rows = min(_MAX_ROWS, max_tokens)
        self.buf_bytes = ((max_tokens + 8) * H * 2 + 255) // 256 * 256
        self.cand_bytes = (size * self.max_rows * 16 + 255) // 256 * 256
        self.vocab = model_cfg.vocab_size
        self.gather_bytes = (_GATHER_ROWS * self.vocab * 4 + 255) // 256 * 256
        total = _CTR_BYTES + 3 * self.buf_bytes + self.cand_bytes + self.gather_bytes
        self.symm = symm_mem.empty(total // 2, dtype=torch.bfloat16, device=device)
        self.symm.zero_()
        torch.cuda.synchronize(device)
        self.hdl = symm_mem.rendezvous(self.symm, dist.group.WORLD)
        self.bases = [int(p) for p in self.hdl.buffer_ptrs]
        assert len(self.bases) == size
        mc = 0
        if USE_MULTIMEM:
            try:
                mc = int(self.hdl.multicast_ptr or 0)
            except Exception as e:  # pragma: no cover - depends on the driver
                log.warning("no NVLS multicast object (%s); using peer loads / stores", e)
        self.mc = mc
        self.in_off = _CTR_BYTES
        self.out_off = _CTR_BYTES + self.buf_bytes
        self.out2_off = _CTR_BYTES + 2 * self.buf_bytes
        self.cand_off = _CTR_BYTES + 3 * self.buf_bytes
        self.gather_off = self.cand_off + self.cand_bytes
        z = lambda n: torch.zeros(n, dtype=torch.int32, device=device)  # noqa: E731
        self.ep_norm, self.ep_ar, self.ep_vocab = z(_RN_BLOCKS), z(_RN_BLOCKS), z(self.max_rows)
        self.ep_gather = z(_GA_BLOCKS)
        dist.barrier()
        log.info("fused TP comm ready: rank %d/%d, %.1f MiB symmetric, %s", rank, size,
                 total / 2**20, "NVLS multimem" if mc else "peer loads/stores")

    # ------------------------------------------------------------ buffers
    def _view(self, off: int, T: int, H: int) -> torch.Tensor:
        return self.symm[off // 2:off // 2 + T * H].view(T, H)

    def reduce_buffer(self, T: int, H: int) -> Optional[torch.Tensor]:
        """This rank's partial-sum buffer: the row-parallel GEMM stores its
        output here (local stores)."""
        if T > self.max_tokens or H != self.H:
            return None
        return self._view(self.in_off, T, H)

    def shard(self, T: int) -> Tuple[int, int]:
        """Token rows [lo, hi) whose residual this rank keeps."""
        return T * self.rank // self.size, T * (self.rank + 1) // self.size

    # ------------------------------------------------------------ reductions
    def reduce_norm(self, T: int, residual: torch.Tensor, w: Optional[torch.Tensor],
                    eps: float) -> torch.Tensor:
        """Sum of every rank's ``in`` rows, plus this rank's residual shard
        (updated in place), RMS-normalised with ``w`` (None: no norm), all
        rows gathered on every rank: returns the [T, H] normalised rows."""
        from .. import ops
        if T == 0:
            return self._view(self.out_off, 0, self.H)
        ops._count(self.C.tp_reduce_norm(self.bases, self.mc, self.rank, self.in_off, self.out_off,
                                         _CTR_NORM, residual, w, float(eps), T, self.H,
                                         self.ep_norm, TIMEOUT_S))
        return self._view(self.out_off, T, self.H)

    def reduce(self, x: torch.Tensor) -> torch.Tensor:
        """Plain all-reduce of a [T, H] tensor (sum over ranks)."""
        T, H = x.shape[0], x.numel() // max(x.shape[0], 1)
        if H != self.H or T > self.max_tokens:
            return super().reduce(x)
        if T == 0:
            return x
        slot = self.reduce_buffer(T, H)
        if x.data_ptr() != slot.data_ptr():
            slot.copy_(x.view(T, H))
        from .. import ops
        ops._count(self.C.tp_reduce_norm(self.bases, self.mc, self.rank, self.in_off, self.out2_off,
                                         _CTR_AR, None, None, 0.0, T, H, self.ep_ar, TIMEOUT_S))
        return self._view(self.out2_off, T, H).view_as(x)

    def linear_reduce(self, x: torch.Tensor, w, b: Optional[torch.Tensor] = None) -> torch.Tensor:
        from .. import ops
        if self.rank != 0:
            b = None
        T = x.shape[0]
        return self.reduce(ops.linear(x, w, b, out=self.reduce_buffer(T, w.shape[0])))

    # ------------------------------------------------------------ sampling
    def gather_vocab(self, x: torch.Tensor) -> torch.Tensor:
        """Full-vocabulary fp32 logits [rows, V] from every rank's slice
        [rows, V/k]: one kernel pushes this rank's slice into every rank's
        gather buffer over NVSwitch (multimem.st) or NVLink peer stores."""
        rows = x.shape[0]
        if (x.dtype != torch.float32 or rows > _GATHER_ROWS or x.shape[-1] * self.size != self.vocab
                or x.shape[-1] % 4):
            return super().gather_vocab(x)
        from .. import ops
        x = x.contiguous()
        ops._count(self.C.tp_gather_vocab(self.bases, self.mc, self.rank, x, self.gather_off,
                                          _CTR_GATHER, self.ep_gather, TIMEOUT_S))
        n = rows * self.vocab
        return self.symm[self.gather_off // 2:self.gather_off // 2 + 2 * n].view(torch.float32).view(
            rows, self.vocab)

    def vocab_greedy(self, logits: torch.Tensor, v0: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Greedy tokens and their log-probabilities over the full vocabulary
        from this rank's fp32 logits slice [rows, V/k] starting at ``v0``;
        every rank gets the same result."""
        from .. import ops
        rows = logits.shape[0]
        if rows > self.max_rows:
            full = self.gather_vocab(logits)
            lp = torch.log_softmax(full, dim=-1)
            tok = full.argmax(-1)
            return tok.int(), lp.gather(1, tok.view(-1, 1)).view(-1)
        tokens = torch.empty(rows, dtype=torch.int32, device=logits.device)
        lps = torch.empty(rows, dtype=torch.float32, device=logits.device)
        ops._count(self.C.tp_vocab_argmax(self.bases, self.mc, self.rank, logits.contiguous(), v0,
                                          self.cand_off, _CTR_VOCAB, tokens, lps, self.ep_vocab,
                                          TIMEOUT_S))
        return tokens, lps

    # ------------------------------------------------------------ lifecycle
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
        self.ep_norm = self.ep_ar = self.ep_vocab = None

    def check(self) -> None:
        st = self.C.read_status(True)
        if st[0] == 2:
            raise CommTimeoutError(f"peer did not arrive within {TIMEOUT_S}s (site {st[1]})")
