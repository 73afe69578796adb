#!/usr/bin/env python3
"""The OpenAI-compatible server and a client of it: starts
`swiftllm-server serve` in a subprocess, then sends a completion, a chat
completion and a streamed chat completion with plain HTTP (no SDK needed).

  python examples/openai_server.py [--model PATH] [--port 8011]
"""

import argparse
import json
import subprocess
import sys
import time
import urllib.request


def post(url: str, body: dict):
    req = urllib.request.Request(url, data=json.dumps(body).encode(),
                                 headers={"Content-Type": "application/json"})
    return urllib.request.urlopen(req, timeout=120)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny-llama")
    ap.add_argument("--port", type=int, default=8011)
    a = ap.parse_args()
    extra = ["--load-format", "dummy"] if a.model.startswith("tiny-") else []
    srv = subprocess.Popen([sys.executable, "-m", "swiftllm_b200.server", "serve", "--model", a.model,
                            "--port", str(a.port), "--max-model-len", "1024"] + extra)
    base = f"http://127.0.0.1:{a.port}"
    try:
        for _ in range(600):
            try:
                urllib.request.urlopen(base + "/health", timeout=1)
                break
            except OSError:
                time.sleep(0.5)
        r = json.load(post(base + "/v1/completions",
                           {"model": a.model, "prompt": "Hello, my name is", "max_tokens": 16}))
        print("completion:", r["choices"][0]["text"])
        r = json.load(post(base + "/v1/chat/completions",
                           {"model": a.model, "max_tokens": 16,
                            "messages": [{"role": "user", "content": "Say hi"}]}))
        print("chat:", r["choices"][0]["message"]["content"])
        with post(base + "/v1/chat/completions",
                  {"model": a.model, "max_tokens": 16, "stream": True,
                   "messages": [{"role": "user", "content": "Count to five"}]}) as resp:
            for line in resp:
                line = line.decode().strip()
                if line.startswith("data: ") and line != "data: [DONE]":
                    delta = json.loads(line[6:])["choices"][0]["delta"].get("content", "")
                    print(delta, end="", flush=True)
        print()
    finally:
        srv.terminate()
        srv.wait(timeout=30)


if __name__ == "__main__":
    main()
