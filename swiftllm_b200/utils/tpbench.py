"""Tensor-parallel row-parallel linear + sum: the fused GEMM -> reduce-scatter
path against GEMM + the separate peer-memory reduction and against cuBLAS +
NCCL, timed with CUDA events (median of 20, max over ranks).

  python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
      -m swiftllm_b200.utils.tpbench [--hidden 4096] [--inner 2048,5504] [--tokens 256,626]
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist


def _time(fn, iters=20):
    for _ in range(3):
        fn()
    ts = []
    for _ in range(iters):
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    ts.sort()
    t = torch.tensor([ts[len(ts) // 2]], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--inner", default="2048,5504")
    ap.add_argument("--tokens", default="1,64,256,626,2048")
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    from ..parallel.comm import build_tp_group, init_distributed
    from ..models.config import ModelConfig
    from .. import ops
    init_distributed(rank, world, "nccl")
    cfg = ModelConfig(hidden_size=a.hidden)
    dev = torch.device("cuda", torch.cuda.current_device())
    tp = build_tp_group(rank, world, dev, "fused", cfg, 8192)
    for K in [int(v) for v in a.inner.split(",")]:
        w = (torch.randn(a.hidden, K, device=dev) * 0.02).bfloat16()
        for T in [int(v) for v in a.tokens.split(",")]:
            x = torch.randn(T, K, device=dev).bfloat16()
            t_fused = _time(lambda: tp.linear_reduce(x, w, fused=True))
            t_unfused = _time(lambda: tp.linear_reduce(x, w, fused=False))
            t_gemm = _time(lambda: ops.linear(x, w, out=tp.reduce_buffer(T, a.hidden)))
            y = torch.empty(T, a.hidden, device=dev, dtype=torch.bfloat16)

            def nccl():
                torch.matmul(x, w.t(), out=y)
                dist.all_reduce(y)
            t_nccl = _time(nccl)
            if rank == 0:
                print(json.dumps({"K": K, "T": T, "fused_ms": round(t_fused, 4),
                                  "unfused_ms": round(t_unfused, 4),
                                  "gemm_only_ms": round(t_gemm, 4),
                                  "cublas_nccl_ms": round(t_nccl, 4)}), flush=True)
    st = tp.C.read_status(True)
    if rank == 0:
        print(json.dumps({"status": list(st)}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
