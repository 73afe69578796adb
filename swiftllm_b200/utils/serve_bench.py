"""Serving load test: Poisson arrivals against the OpenAI-compatible server.

  python -m swiftllm_b200.utils.serve_bench --model llama-3-8b --rates 1,4,16,64 \
      [--requests 2000] [--url http://host:port]   # no --url: start the native server in-process

Workload (the server load-test shape): prompt lengths lognormal with median
512 clipped to [32, 4096], output lengths lognormal with median 128 clipped
to [16, 1024], random token ids, temperature 0.7, top_p 0.9, EOS ignored so
every request produces its drawn length. Requests are streaming
``/v1/completions`` calls with the prompt given as token ids (chat requests
carry text, which a random-token workload does not have).

Per request, on the client: TTFT = first SSE event with generated text or a
finish reason after sending the request; TPOT = (last event - first event) /
(output tokens - 1). Reports p50 / p99 TTFT and TPOT, request throughput and
output tokens/s per rate. Client threads issue requests at the drawn
arrival times; a request that has not finished after --timeout seconds
counts as failed.
"""

from __future__ import annotations

import argparse
import http.client
import json
import math
import threading
import time
from typing import Dict, List, Optional
from urllib.parse import urlparse

import numpy as np


def workload(n: int, seed: int = 0, vocab: int = 32000):
    rng = np.random.default_rng(seed)
    p_len = np.clip(np.round(rng.lognormal(math.log(512), 0.6, n)), 32, 4096).astype(int)
    o_len = np.clip(np.round(rng.lognormal(math.log(128), 0.6, n)), 16, 1024).astype(int)
    prompts = [rng.integers(0, vocab, size=int(p)).tolist() for p in p_len]
    return prompts, o_len.tolist()


def _one(host: str, port: int, key: Optional[str], prompt: List[int], out_len: int,
         res: Dict, timeout: float) -> None:
    body = json.dumps({"prompt": prompt, "max_tokens": int(out_len), "temperature": 0.7,
                       "top_p": 0.9, "stream": True, "ignore_eos": True})
    hdr = {"Content-Type": "application/json"}
    if key:
        hdr["Authorization"] = f"Bearer {key}"
    t0 = time.perf_counter()
    first = last = None
    try:
        c = http.client.HTTPConnection(host, port, timeout=timeout)
        c.request("POST", "/v1/completions", body=body, headers=hdr)
        r = c.getresponse()
        if r.status != 200:
            res["error"] = r.status
            return
        buf = b""
        while True:
            chunk = r.read1(65536) if hasattr(r, "read1") else r.read(4096)
            if not chunk:
                break
            buf += chunk
            while b"\n\n" in buf:
                ev, buf = buf.split(b"\n\n", 1)
                if not ev.startswith(b"data: "):
                    continue
                data = ev[6:]
                now = time.perf_counter()
                if data == b"[DONE]":
                    continue
                if first is None:
                    first = now
                last = now
        c.close()
    except Exception as e:  # counted as failed
        res["error"] = repr(e)
        return
    if first is None:
        res["error"] = "no events"
        return
    res["ttft"] = first - t0
    res["tpot"] = (last - first) / max(out_len - 1, 1)
    res["e2e"] = last - t0
    res["out"] = out_len


def run_rate(url_host: str, port: int, key: Optional[str], rate: float, prompts, outs,
             timeout: float, seed: int = 1) -> Dict:
    rng = np.random.default_rng(seed)
    gaps = rng.exponential(1.0 / rate, len(prompts))
    arrivals = np.cumsum(gaps) - gaps[0]
    results = [dict() for _ in prompts]
    threads = []
    t0 = time.perf_counter()
    for i, (p, o) in enumerate(zip(prompts, outs)):
        wait = t0 + arrivals[i] - time.perf_counter()
        if wait > 0:
            time.sleep(wait)
        th = threading.Thread(target=_one, args=(url_host, port, key, p, o, results[i], timeout),
                              daemon=True)
        th.start()
        threads.append(th)
    for th in threads:
        th.join(timeout)
    wall = time.perf_counter() - t0
    ok = [r for r in results if "ttft" in r]
    ttft = np.array([r["ttft"] for r in ok]) * 1e3
    tpot = np.array([r["tpot"] for r in ok]) * 1e3
    pct = lambda a, q: round(float(np.percentile(a, q)), 2) if a.size else None  # noqa: E731
    return {"rate_req_s": rate, "requests": len(prompts), "completed": len(ok),
            "failed": len(prompts) - len(ok), "wall_s": round(wall, 2),
            "throughput_req_s": round(len(ok) / wall, 3),
            "output_tok_s": round(sum(r["out"] for r in ok) / wall, 1),
            "ttft_ms_p50": pct(ttft, 50), "ttft_ms_p99": pct(ttft, 99),
            "tpot_ms_p50": pct(tpot, 50), "tpot_ms_p99": pct(tpot, 99)}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3-8b")
    ap.add_argument("--rates", default="1,4,16,64")
    ap.add_argument("--requests", type=int, default=2000)
    ap.add_argument("--url", default=None)
    ap.add_argument("--api-key", default=None)
    ap.add_argument("--timeout", type=float, default=600.0)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--max-model-len", type=int, default=5120)
    a = ap.parse_args(argv)
    srv = None
    vocab = 32000
    if a.url:
        u = urlparse(a.url)
        host, port = u.hostname, u.port or 80
    else:
        from ..config import ServerConfig
        from ..engine.llm import LLM
        from ..server.native_server import NativeServer
        llm = LLM(a.model, load_format="dummy", dtype="auto", tensor_parallel_size=a.tp,
                  max_model_len=a.max_model_len, enable_chunked_prefill=True,
                  gpu_memory_utilization=0.9)
        srv = NativeServer(llm, ServerConfig(host="127.0.0.1", port=0)).start()
        host, port = "127.0.0.1", srv.port
        vocab = llm.llm_engine.model_config.vocab_size
    out = []
    for i, rate in enumerate(float(r) for r in a.rates.split(",")):
        prompts, outs = workload(a.requests, seed=i, vocab=vocab)
        r = run_rate(host, port, a.api_key, rate, prompts, outs, a.timeout, seed=100 + i)
        r.update(model=a.model, tp=a.tp, frontend="native" if srv else a.url)
        print(json.dumps(r), flush=True)
        out.append(r)
    if srv is not None:
        srv.stop()


if __name__ == "__main__":
    main()
