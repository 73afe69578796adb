#!/usr/bin/env python3
"""Token streaming with AsyncLLM: text arrives as it is generated, several
requests interleaved on one engine.

  python examples/streaming.py [--model PATH]
"""

import argparse
import asyncio

from swiftllm_b200 import AsyncLLM, SamplingParams


async def stream_one(llm: AsyncLLM, tag: str, prompt: str, sp: SamplingParams) -> None:
    seen = 0
    async for out in llm.generate(prompt, sp):
        text = out.outputs[0].text
        if len(text) > seen:
            print(f"[{tag}] {text[seen:]!r}", flush=True)
            seen = len(text)
        if out.finished:
            print(f"[{tag}] done: {out.outputs[0].finish_reason}")


async def main_async(model: str) -> None:
    dummy = model.startswith("tiny-")
    llm = AsyncLLM(model, load_format="dummy" if dummy else "auto", max_model_len=1024)
    sp = SamplingParams(temperature=0.8, top_p=0.95, max_tokens=24, seed=0)
    await asyncio.gather(stream_one(llm, "a", "Once upon a time", sp),
                         stream_one(llm, "b", "The three laws of robotics are", sp))
    llm.shutdown()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny-llama")
    asyncio.run(main_async(ap.parse_args().model))


if __name__ == "__main__":
    main()
