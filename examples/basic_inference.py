#!/usr/bin/env python3
"""Offline generation with the LLM API: one prompt, a batch, and per-prompt
sampling parameters.

  python examples/basic_inference.py                       # random-init tiny model
  python examples/basic_inference.py --model /path/to/Llama-2-7b-hf
"""

import argparse

from swiftllm_b200 import LLM, SamplingParams


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny-llama")
    ap.add_argument("--tp", type=int, default=1, help="tensor_parallel_size")
    a = ap.parse_args()
    dummy = a.model.startswith("tiny-")
    llm = LLM(a.model, tensor_parallel_size=a.tp, gpu_memory_utilization=0.9,
              load_format="dummy" if dummy else "auto", max_model_len=1024)
    sp = SamplingParams(temperature=0.7, top_p=0.9, max_tokens=64, stop=["\n\n"], seed=0)

    out = llm.generate("What is the capital of France?", sp)[0]
    print("single:", repr(out.outputs[0].text))

    prompts = ["Explain quantum computing in simple terms:",
               "Write a haiku about artificial intelligence:",
               "Describe the process of photosynthesis:"]
    for o in llm.generate(prompts, sp):
        print(f"batch: {o.prompt!r} -> {o.outputs[0].text!r}")

    # one SamplingParams per prompt: greedy for the first, sampled for the second
    per = [SamplingParams(temperature=0.0, max_tokens=32),
           SamplingParams(temperature=1.0, top_k=50, max_tokens=32, seed=1)]
    for o in llm.generate(prompts[:2], per):
        print(f"per-prompt: {o.outputs[0].text!r} ({o.outputs[0].finish_reason})")
    llm.shutdown()


if __name__ == "__main__":
    main()
