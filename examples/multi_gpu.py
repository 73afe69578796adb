#!/usr/bin/env python3
"""Tensor parallelism: the same model split over 1, 2, 4 ... GPUs of one
node (one process per GPU, spawned by the engine; the row-parallel sums run
in the fused NVLink kernels, comm_backend="nccl" selects the library
baseline).

  python examples/multi_gpu.py --tp 1,2,4 [--model PATH] [--comm fused|nccl]
"""

import argparse
import time

import torch

from swiftllm_b200 import LLM, SamplingParams


def run(model: str, tp: int, comm: str, n_req: int, max_tokens: int) -> float:
    dummy = model.startswith("tiny-") or model.startswith("llama-")
    llm = LLM(model, tensor_parallel_size=tp, comm_backend=comm,
              load_format="dummy" if dummy else "auto", max_model_len=2048)
    sp = SamplingParams(temperature=0.0, max_tokens=max_tokens, ignore_eos=True)
    prompts = [[(7 * i + j) % 1000 + 1 for j in range(128)] for i in range(n_req)]
    llm.generate(prompt_token_ids=prompts[:2], sampling_params=sp, use_tqdm=False)
    t0 = time.perf_counter()
    outs = llm.generate(prompt_token_ids=prompts, sampling_params=sp, use_tqdm=False)
    dt = time.perf_counter() - t0
    llm.shutdown()
    return sum(len(o.outputs[0].token_ids) for o in outs) / dt


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny-llama")
    ap.add_argument("--tp", default="1,2")
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"])
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--max-tokens", type=int, default=128)
    a = ap.parse_args()
    sizes = [int(v) for v in a.tp.split(",") if int(v) <= max(torch.cuda.device_count(), 1)]
    base = None
    for tp in sizes:
        tps = run(a.model, tp, a.comm, a.requests, a.max_tokens)
        base = base or tps
        print(f"tp={tp}: {tps:10.1f} output tok/s  speedup {tps / base:.2f}x")


if __name__ == "__main__":
    main()
