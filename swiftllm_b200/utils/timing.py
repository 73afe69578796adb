"""Device timing: CUDA events per rank, reduced to the max over ranks.

Rule used everywhere a number is reported: warm up, synchronise, record an
event on the launching stream, run, record, synchronise, and take the max
of the per-rank elapsed times (all-reduce MAX over the process group)."""

from __future__ import annotations

import json
import os
from typing import Optional

import torch


class DeviceTimer:
    def __init__(self, device=None):
        self.device = device
        self.start = torch.cuda.Event(enable_timing=True)
        self.end = torch.cuda.Event(enable_timing=True)

    def __enter__(self):
        torch.cuda.synchronize(self.device)
        self.start.record()
        return self

    def __exit__(self, *exc):
        self.end.record()
        torch.cuda.synchronize(self.device)
        self.ms = self.start.elapsed_time(self.end)
        return False


def max_over_ranks(value: float, group=None) -> float:
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return value
    dev = "cuda" if torch.cuda.is_available() and dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def measured_peaks(path: Optional[str] = None) -> dict:
    """Roofline denominators: the driver-measured copy bandwidth and cuBLAS
    bf16 rate, else the pool's earlier measurement."""
    here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    path = path or os.path.join(here, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        d["source"] = "measured"
        return d
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                "source": "fallback"}
