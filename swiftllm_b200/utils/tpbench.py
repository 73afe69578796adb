"""Tensor-parallel row-parallel linear + cross-rank sum + residual add +
RMSNorm, the unit that closes every attention and MLP block: our GEMM into
the symmetric buffer plus the one-kernel NVLS / peer reduction
(``tp.reduce_norm``) against cuBLAS + NCCL all-reduce + the fused add-norm
kernel. CUDA events, median of 20, max over ranks. Also reports the
reduction alone and its fraction of the NVLink roofline: bytes each GPU must
move per direction, (k-1)/k * T * H * 2, at the measured 770 GB/s.

  python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
      -m swiftllm_b200.utils.tpbench [--hidden 4096] [--inner 2048,5504] [--tokens 256,626]
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0  # measured NVLink peer copy per direction on this pool's B200s


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


def _time_graph(fn, reps=20):
    """Per-call time of ``reps`` back-to-back calls captured in one CUDA
    graph (ranks stay in lock step through the collectives, so one-off
    launch skew between ranks is excluded); max over ranks."""
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            for _ in range(reps):
                fn()
    torch.cuda.current_stream().wait_stream(st)
    g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / reps], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--inner", default="2048,5504")
    ap.add_argument("--tokens", default="1,64,256,832,2048,8192")
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    from ..parallel.comm import build_tp_group, init_distributed
    from ..models.config import ModelConfig
    from .. import ops
    init_distributed(rank, world, "nccl")
    cfg = ModelConfig(hidden_size=a.hidden)
    dev = torch.device("cuda", torch.cuda.current_device())
    H = a.hidden
    tp = build_tp_group(rank, world, dev, "fused", cfg, 8192)
    nw = torch.ones(H, device=dev, dtype=torch.bfloat16)
    for K in [int(v) for v in a.inner.split(",")]:
        w = (torch.randn(H, K, device=dev) * 0.02).bfloat16()
        for T in [int(v) for v in a.tokens.split(",")]:
            x = torch.randn(T, K, device=dev).bfloat16()
            res = torch.randn(T, H, device=dev).bfloat16()

            def ours():
                ops.linear(x, w, out=tp.reduce_buffer(T, H))
                tp.reduce_norm(T, res, nw, 1e-5)
            t_ours = _time(ours)
            t_comm = _time(lambda: tp.reduce_norm(T, res, nw, 1e-5))
            t_gemm = _time(lambda: ops.linear(x, w, out=tp.reduce_buffer(T, H)))
            y = torch.empty(T, H, device=dev, dtype=torch.bfloat16)

            def nccl():
                torch.matmul(x, w.t(), out=y)
                dist.all_reduce(y)
                ops.rms_norm(y, nw, 1e-5, res)
            t_nccl = _time(nccl)
            t_cublas = _time(lambda: torch.matmul(x, w.t(), out=y))
            # back to back in a graph, as inside a decode step
            g_comm = _time_graph(lambda: tp.reduce_norm(T, res, nw, 1e-5))
            g_ours = _time_graph(ours)
            g_nccl = _time_graph(nccl)
            link_s = (world - 1) / world * T * H * 2 / (LINK_GBS * 1e9)
            if rank == 0:
                print(json.dumps({"K": K, "T": T, "ours_ms": round(t_ours, 4),
                                  "reduce_norm_ms": round(t_comm, 4),
                                  "gemm_ms": round(t_gemm, 4),
                                  "cublas_nccl_norm_ms": round(t_nccl, 4),
                                  "cublas_ms": round(t_cublas, 4),
                                  "graph_reduce_norm_ms": round(g_comm, 4),
                                  "graph_ours_ms": round(g_ours, 4),
                                  "graph_cublas_nccl_norm_ms": round(g_nccl, 4),
                                  "reduce_link_roofline_frac": round(link_s * 1e3 / t_comm, 3),
                                  "multimem": bool(tp.mc)}), flush=True)
    st = tp.C.read_status(True)
    if rank == 0:
        print(json.dumps({"status": list(st)}), flush=True)
    tp.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
