"""Tensor-parallel communication.

Two backends behind the model's ``TPGroup`` interface:

* ``nccl`` (the baseline to beat): torch.distributed all-reduce after every
  row-parallel GEMM and all-gather of vocab-parallel logits.
* ``fused`` (the product): the reduction after o_proj / down_proj runs in
  our own kernel over NVLink peer memory (symmetric buffers rendezvoused
  through torch.distributed._symmetric_memory): each rank publishes its
  partial, a flag with a bounded wait orders the exchange, and the reducing
  kernel sums the partials (fixed rank order, fp32) into the replicated
  residual stream. Falls back to NCCL only on CPU (gloo) process groups.

Parity: crates/swiftllm-core/src/execution/tensor_parallel.rs
(CommunicationBackend Nccl | Gloo | Custom :55-63, all_reduce /
all_gather / reduce_scatter stubs :115-141, ReduceOp :218-230).
"""

from __future__ import annotations

import os
from typing import Optional

import torch

from ..models.decoder import TPGroup
from ..utils.logging import get_logger

log = get_logger(__name__)


def init_distributed(rank: int, world: int, backend: str) -> None:
    import torch.distributed as dist
    if dist.is_initialized():
        return
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29511")
    kwargs = {}
    if backend == "nccl":
        kwargs["device_id"] = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group(backend=backend, rank=rank, world_size=world, **kwargs)


def teardown_distributed() -> None:
    """Orderly end of a multi-rank job: every rank calls this after its
    engine / worker released its device buffers; a barrier makes sure no
    peer still reads them, then the process group is destroyed so the
    interpreter exits normally."""
    import torch.distributed as dist
    if not dist.is_initialized():
        return
    if torch.cuda.is_available():
        torch.cuda.synchronize()
    try:
        dist.barrier()
    finally:
        dist.destroy_process_group()


class NcclTP(TPGroup):
    """torch.distributed collectives (NCCL on GPUs, gloo on CPU)."""

    def __init__(self, rank: int, size: int):
        super().__init__(rank, size)
        import torch.distributed as dist
        self.dist = dist

    def reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.size > 1:
            self.dist.all_reduce(x)
        return x

    def gather_vocab(self, x: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return x
        parts = [torch.empty_like(x) for _ in range(self.size)]
        self.dist.all_gather(parts, x.contiguous())
        return torch.cat(parts, dim=-1)


def build_tp_group(rank: int, world: int, device: torch.device, backend: str,
                   model_cfg=None, max_tokens: int = 8192) -> TPGroup:
    if world == 1:
        return TPGroup(0, 1)
    if backend == "fused" and device.type == "cuda":
        from .fused_comm import FusedTP
        return FusedTP(rank, world, device, model_cfg, max_tokens)
    return NcclTP(rank, world)
