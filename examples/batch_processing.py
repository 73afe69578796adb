#!/usr/bin/env python3
"""Throughput of offline continuous batching as the batch grows: the same
prompts submitted in batches of 1..32, output tokens per second of each.

  python examples/batch_processing.py [--model PATH] [--max-tokens 64]
"""

import argparse
import time

from swiftllm_b200 import LLM, SamplingParams


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny-llama")
    ap.add_argument("--max-tokens", type=int, default=64)
    a = ap.parse_args()
    dummy = a.model.startswith("tiny-")
    llm = LLM(a.model, load_format="dummy" if dummy else "auto", max_model_len=1024,
              max_num_seqs=64)
    sp = SamplingParams(temperature=0.0, max_tokens=a.max_tokens, ignore_eos=True)
    llm.generate(["warm up"], sp)
    for bs in (1, 2, 4, 8, 16, 32):
        prompts = [f"Request {i}: summarise the history of computing." for i in range(bs)]
        t0 = time.perf_counter()
        outs = llm.generate(prompts, sp, use_tqdm=False)
        dt = time.perf_counter() - t0
        n = sum(len(o.outputs[0].token_ids) for o in outs)
        print(f"batch {bs:3d}: {n / dt:10.1f} output tok/s  ({dt * 1e3:.1f} ms)")
    print(llm.llm_engine.stats())
    llm.shutdown()


if __name__ == "__main__":
    main()
