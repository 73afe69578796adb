"""``swiftllm`` command line.

Subcommands and flags follow python/swiftllm/cli.py:45-441 (serve,
generate, benchmark, convert, info, chat, download) and the Rust binary's
serve flags (crates/swiftllm-server/src/main.rs:37-150). Additions:
``--load-format dummy`` (random-init presets), ``--max-num-seqs``,
``--comm-backend``, ``--enforce-eager``. ``convert`` is implemented (the
reference leaves it TODO, cli.py:734-745): GGUF or safetensors in,
safetensors with HF tensor names out, in the requested dtype.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from typing import List, Optional

from . import __version__


def _engine_args(p: argparse.ArgumentParser) -> None:
    p.add_argument("-m", "--model", required=True)
    p.add_argument("--tensor-parallel-size", "-tp", type=int, default=1)
    p.add_argument("--max-model-len", type=int, default=None)
    p.add_argument("--gpu-memory-utilization", type=float, default=0.90)
    p.add_argument("--dtype", default="auto")
    p.add_argument("--quantization", "-q", default=None)
    p.add_argument("--trust-remote-code", action="store_true")
    p.add_argument("--download-dir", default=None)
    p.add_argument("--load-format", default="auto")
    p.add_argument("--max-num-seqs", type=int, default=256)
    p.add_argument("--block-size", type=int, default=16)
    p.add_argument("--swap-space", type=float, default=4.0)
    p.add_argument("--enable-prefix-caching", action="store_true")
    p.add_argument("--enable-chunked-prefill", action="store_true")
    p.add_argument("--speculative-model", default=None)
    p.add_argument("--num-speculative-tokens", type=int, default=5)
    p.add_argument("--comm-backend", default="fused", choices=["fused", "nccl"])
    p.add_argument("--enforce-eager", action="store_true")
    p.add_argument("--seed", type=int, default=0)


def _engine_kwargs(a) -> dict:
    kw = dict(tensor_parallel_size=a.tensor_parallel_size, max_model_len=a.max_model_len,
              gpu_memory_utilization=a.gpu_memory_utilization, dtype=a.dtype,
              quantization=a.quantization, trust_remote_code=a.trust_remote_code,
              download_dir=a.download_dir, seed=a.seed)
    for k in ("load_format", "max_num_seqs", "block_size", "swap_space", "enable_prefix_caching",
              "enable_chunked_prefill", "speculative_model", "num_speculative_tokens",
              "comm_backend", "enforce_eager"):
        if hasattr(a, k):
            kw[k] = getattr(a, k)
    return kw


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="swiftllm", description="B200-native LLM inference engine")
    p.add_argument("--version", action="version", version=f"swiftllm_b200 {__version__}")
    sub = p.add_subparsers(dest="command")
    s = sub.add_parser("serve", help="Start the OpenAI-compatible server")
    _engine_args(s)
    s.add_argument("--host", default="0.0.0.0")
    s.add_argument("-p", "--port", type=int, default=8000)
    s.add_argument("--api-key", default=None)
    s.add_argument("--served-model-name", default=None)
    s.add_argument("--frontend", choices=["native", "fastapi"], default="native",
                   help="native: C++ HTTP/SSE front end driving the engine directly; "
                        "fastapi: ASGI app over AsyncLLM")
    g = sub.add_parser("generate", help="Run offline generation")
    _engine_args(g)
    g.add_argument("-p", "--prompt", action="append", default=None)
    g.add_argument("-f", "--file", default=None)
    g.add_argument("--max-tokens", type=int, default=256)
    g.add_argument("--temperature", type=float, default=0.7)
    g.add_argument("--top-p", type=float, default=1.0)
    g.add_argument("--top-k", type=int, default=-1)
    g.add_argument("-n", "--num-sequences", type=int, default=1)
    g.add_argument("-o", "--output", default=None)
    g.add_argument("--json", action="store_true")
    b = sub.add_parser("benchmark", help="Throughput / latency benchmark")
    _engine_args(b)
    b.add_argument("--input-len", type=int, default=512)
    b.add_argument("--output-len", type=int, default=128)
    b.add_argument("--num-prompts", type=int, default=100)
    b.add_argument("--concurrency", type=int, default=0)
    b.add_argument("--warmup", type=int, default=1)
    b.add_argument("-o", "--output", default=None)
    c = sub.add_parser("convert", help="Convert GGUF / safetensors to safetensors")
    c.add_argument("-i", "--input", required=True)
    c.add_argument("-o", "--output", required=True)
    c.add_argument("--format", default="safetensors", choices=["safetensors"])
    c.add_argument("--dtype", default="bfloat16", choices=["bfloat16", "float16", "float32"])
    c.add_argument("--quantize", default=None)
    c.add_argument("--calibration-data", default=None)
    i = sub.add_parser("info", help="Show model information")
    i.add_argument("-m", "--model", required=True)
    i.add_argument("--json", action="store_true")
    i.add_argument("--download-dir", default=None)
    ch = sub.add_parser("chat", help="Interactive chat")
    _engine_args(ch)
    ch.add_argument("--system", default=None)
    ch.add_argument("--max-tokens", type=int, default=256)
    ch.add_argument("--temperature", type=float, default=0.7)
    d = sub.add_parser("download", help="Download a model from the HF hub")
    d.add_argument("-m", "--model", required=True)
    d.add_argument("--download-dir", default=None)
    d.add_argument("--revision", default=None)
    d.add_argument("--token", default=None)
    return p


def cmd_serve(a) -> int:
    from .config import ServerConfig
    cfg = ServerConfig(host=a.host, port=a.port, api_key=a.api_key,
                       served_model_name=a.served_model_name)
    if getattr(a, "frontend", "native") == "native":
        from .engine.llm import LLM
        from .server.native_server import serve_native
        serve_native(LLM(a.model, **_engine_kwargs(a)), cfg)
        return 0
    from .engine.llm import AsyncLLM
    from .server.openai_server import serve
    serve(AsyncLLM(a.model, **_engine_kwargs(a)), cfg)
    return 0


def cmd_generate(a) -> int:
    from . import LLM, SamplingParams
    prompts: List[str] = list(a.prompt or [])
    if a.file:
        with open(a.file) as f:
            prompts += [ln.rstrip("\n") for ln in f if ln.strip()]
    if not prompts:
        print("no prompts given (-p or -f)", file=sys.stderr)
        return 2
    llm = LLM(a.model, **_engine_kwargs(a))
    sp = SamplingParams(temperature=a.temperature, top_p=a.top_p, top_k=a.top_k,
                        max_tokens=a.max_tokens, n=a.num_sequences)
    outs = llm.generate(prompts, sp, use_tqdm=False)
    res = [{"prompt": o.prompt, "outputs": [c.text for c in o.outputs],
            "finish_reasons": [c.finish_reason.value if c.finish_reason else None
                               for c in o.outputs]} for o in outs]
    text = json.dumps(res, indent=2) if a.json else "\n".join(
        f"{r['prompt']!r} -> {r['outputs'][0]!r}" for r in res)
    if a.output:
        with open(a.output, "w") as f:
            f.write(text)
    else:
        print(text)
    return 0


def cmd_benchmark(a) -> int:
    """Same metrics as python/swiftllm/cli.py:662-731: throughput =
    (input + output tokens) / elapsed, latency per token, requests/s; plus
    output tok/s and p50 TTFT / TPOT from the engine's per-request metrics."""
    import numpy as np
    from . import LLM, SamplingParams
    llm = LLM(a.model, **_engine_kwargs(a))
    rng = np.random.default_rng(a.seed)
    vocab = llm.llm_engine.model_config.vocab_size if llm.llm_engine.model_config else 32000
    llm.llm_engine._ensure_initialized()
    vocab = llm.llm_engine.model_config.vocab_size
    prompts = [rng.integers(0, vocab, size=a.input_len).tolist() for _ in range(a.num_prompts)]
    sp = SamplingParams(temperature=0.0, max_tokens=a.output_len, ignore_eos=True)
    for _ in range(a.warmup):
        llm.generate(prompt_token_ids=prompts[:2], sampling_params=sp, use_tqdm=False)
    t0 = time.perf_counter()
    outs = llm.generate(prompt_token_ids=prompts, sampling_params=sp, use_tqdm=False)
    el = time.perf_counter() - t0
    n_out = sum(len(o.outputs[0].token_ids) for o in outs)
    n_in = sum(len(p) for p in prompts)
    ttft = [o.metrics["ttft"] for o in outs if o.metrics.get("ttft") is not None]
    tpot = [o.metrics["tpot"] for o in outs if o.metrics.get("tpot") is not None]
    res = {"elapsed_s": el, "requests_per_s": len(outs) / el,
           "throughput_tokens_per_s": (n_in + n_out) / el, "output_tokens_per_s": n_out / el,
           "latency_per_token_ms": el / max(n_out, 1) * 1e3,
           "p50_ttft_ms": float(np.median(ttft)) * 1e3 if ttft else None,
           "p50_tpot_ms": float(np.median(tpot)) * 1e3 if tpot else None}
    text = json.dumps(res, indent=2)
    if a.output:
        with open(a.output, "w") as f:
            f.write(text)
    print(text)
    return 0


def cmd_convert(a) -> int:
    from .loaders.convert import convert
    n = convert(a.input, a.output, a.dtype)
    print(f"wrote {n} tensors to {a.output}")
    return 0


def cmd_info(a) -> int:
    from .model_resolver import resolve_model
    from .models.config import load_config
    path = resolve_model(a.model, a.download_dir)
    cfg = load_config(path)
    d = cfg.to_dict()
    d["num_params"] = cfg.num_params()
    d["kv_cache_bytes_per_token_bf16"] = cfg.kv_cache_bytes_per_token(2)
    if a.json:
        print(json.dumps(d, indent=2))
    else:
        for k, v in d.items():
            print(f"{k:>30}: {v}")
    return 0


def cmd_chat(a) -> int:
    from . import LLM, SamplingParams
    from .engine.tokenizer import chat_prompt
    llm = LLM(a.model, **_engine_kwargs(a))
    msgs = [{"role": "system", "content": a.system}] if a.system else []
    sp = SamplingParams(temperature=a.temperature, max_tokens=a.max_tokens)
    while True:
        try:
            line = input("You: ")
        except (EOFError, KeyboardInterrupt):
            print()
            return 0
        if line.strip() in ("/exit", "/quit"):
            return 0
        msgs.append({"role": "user", "content": line})
        out = llm.generate([chat_prompt(msgs)], sp, use_tqdm=False)[0].outputs[0].text
        print(f"Assistant: {out}")
        msgs.append({"role": "assistant", "content": out})


def cmd_download(a) -> int:
    from .model_resolver import resolve_model
    print(resolve_model(a.model, a.download_dir, a.token))
    return 0


def main(argv: Optional[List[str]] = None) -> int:
    p = build_parser()
    a = p.parse_args(argv)
    if not a.command:
        p.print_help()
        return 0
    return {"serve": cmd_serve, "generate": cmd_generate, "benchmark": cmd_benchmark,
            "convert": cmd_convert, "info": cmd_info, "chat": cmd_chat,
            "download": cmd_download}[a.command](a)


if __name__ == "__main__":
    sys.exit(main())
