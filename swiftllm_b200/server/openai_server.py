"""OpenAI-compatible HTTP server (FastAPI + uvicorn) over AsyncLLM.

Routes (parity with crates/swiftllm-server/src/lib.rs:46-61 and the
Python CLI server python/swiftllm/cli.py:476-579):
  GET  /health, /v1/health          {"status": "ok", "version": ...}
  GET  /v1/models, /v1/models/{id}
  POST /v1/chat/completions         streaming (SSE) and non-streaming
  POST /v1/completions              streaming (SSE) and non-streaming
  GET  /metrics                     scheduler / memory / execution counters
Schemas follow crates/swiftllm-server/src/api/openai.rs:25-320 (request
fields temperature, top_p, n, stream, stop, max_tokens (default 256),
presence/frequency penalty, seed, logprobs, top_logprobs; ids
"chatcmpl-<24 hex>" and "cmpl-<24 hex>"). Unlike the reference, handlers run
the engine: prompt tokens come from the tokenizer, streamed deltas are real
tokens, ``usage`` counts real tokens and ``finish_reason`` is stop / length.
When ``api_key`` is set, requests need ``Authorization: Bearer <key>`` (the
reference stores the key and never checks it, lib.rs:27-35).
"""

from __future__ import annotations

import json
import time
import uuid
from typing import Any, Dict, List, Optional, Union

from ..config import SamplingParams, ServerConfig

try:  # module level: FastAPI resolves the (string) annotations against globals
    from fastapi import Request
except ImportError:  # pragma: no cover - server extra not installed
    Request = None
from ..engine.tokenizer import chat_prompt

VERSION = "0.1.0"


def _sampling(req: Dict[str, Any], default_max: int = 256) -> SamplingParams:
    stop = req.get("stop")
    if isinstance(stop, str):
        stop = [stop]
    lp = req.get("logprobs")
    top_lp = req.get("top_logprobs")
    if isinstance(lp, bool):
        lp = (top_lp or 1) if lp else None
    return SamplingParams(
        temperature=float(req.get("temperature", 1.0)),
        top_p=float(req.get("top_p", 1.0)),
        top_k=int(req.get("top_k", -1)),
        min_p=float(req.get("min_p", 0.0)),
        n=int(req.get("n", 1)),
        max_tokens=int(req.get("max_tokens") or default_max),
        stop=stop,
        presence_penalty=float(req.get("presence_penalty", 0.0)),
        frequency_penalty=float(req.get("frequency_penalty", 0.0)),
        repetition_penalty=float(req.get("repetition_penalty", 1.0)),
        seed=req.get("seed"),
        logprobs=lp,
        ignore_eos=bool(req.get("ignore_eos", False)),
        min_tokens=int(req.get("min_tokens", 0)),
    )


def create_app(llm, config: Optional[ServerConfig] = None):
    from fastapi import FastAPI
    from fastapi.middleware.cors import CORSMiddleware
    from fastapi.responses import JSONResponse, StreamingResponse

    cfg = config or ServerConfig()
    model_name = cfg.served_model_name or llm.config.model
    app = FastAPI(title="swiftllm_b200", version=VERSION, root_path=cfg.root_path)
    app.add_middleware(CORSMiddleware, allow_origins=cfg.cors_allow_origins,
                       allow_methods=["GET", "POST", "OPTIONS"],
                       allow_headers=["Content-Type", "Authorization"])

    def err(status: int, msg: str, kind: str = "invalid_request_error"):
        return JSONResponse(status_code=status,
                            content={"error": {"message": msg, "type": kind, "code": status}})

    @app.middleware("http")
    async def auth(request: Request, call_next):
        if cfg.api_key and request.url.path.startswith("/v1") and request.url.path != "/v1/health":
            if request.headers.get("authorization", "") != f"Bearer {cfg.api_key}":
                return err(401, "invalid or missing API key", "authentication_error")
        return await call_next(request)

    @app.get("/health")
    @app.get("/v1/health")
    async def health():
        return {"status": "ok", "version": VERSION}

    def model_card():
        return {"id": model_name, "object": "model", "created": int(time.time()),
                "owned_by": "swiftllm"}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [model_card()]}

    @app.get("/v1/models/{model_id:path}")
    async def get_model(model_id: str):
        if model_id != model_name:
            return err(404, f"model {model_id!r} not found", "not_found_error")
        return model_card()

    @app.get("/metrics")
    async def metrics():
        s = llm.stats()
        return {
            "scheduler": {"running_requests": s.get("num_running", 0),
                          "waiting_requests": s.get("num_waiting", 0),
                          "completed_requests": s.get("completed_requests", 0),
                          "throughput_tps": s.get("throughput_tps", 0.0)},
            "memory": {"gpu_utilization": s.get("gpu_block_utilization", 0.0),
                       "cpu_utilization": s.get("cpu_block_utilization", 0.0),
                       "free_gpu_blocks": s.get("free_gpu_blocks", 0),
                       "free_cpu_blocks": s.get("free_cpu_blocks", 0)},
            "execution": {"prefill_tokens": s.get("prefill_tokens", 0),
                          "decode_tokens": s.get("decode_tokens", 0),
                          "total_forward_passes": s.get("forward_passes", 0)},
        }

    async def run(prompt: Optional[str], ids: Optional[List[int]], sp: SamplingParams,
                  rid: str, request: Request):
        final = None
        async for out in llm.generate(prompt, sp, request_id=rid, prompt_token_ids=ids):
            final = out
            if await request.is_disconnected():
                await llm.abort(rid)
                break
        return final

    def usage(out) -> Dict[str, int]:
        p = len(out.prompt_token_ids)
        c = sum(len(o.token_ids) for o in out.outputs)
        return {"prompt_tokens": p, "completion_tokens": c, "total_tokens": p + c}

    def finish(o) -> Optional[str]:
        return o.finish_reason.value if o.finish_reason is not None else None

    def prompt_of(req) -> (Optional[str], Optional[List[int]]):
        p = req.get("prompt", "")
        if isinstance(p, list):
            if p and isinstance(p[0], int):
                return None, p
            p = p[0] if p else ""
        return p, None

    def sse(obj) -> str:
        return f"data: {json.dumps(obj)}\n\n"

    @app.post("/v1/chat/completions")
    async def chat(request: Request):
        try:
            req = await request.json()
            sp = _sampling(req)
            msgs = req["messages"]
        except Exception as e:  # malformed request
            return err(400, f"bad request: {e}")
        tok = llm.engine.tokenizer
        if hasattr(tok, "apply_chat_template") and getattr(tok, "chat_template", None):
            prompt = tok.apply_chat_template(msgs, add_generation_prompt=True, tokenize=False)
        else:
            prompt = chat_prompt(msgs)
        rid = f"chatcmpl-{uuid.uuid4().hex[:24]}"
        created = int(time.time())
        if req.get("stream"):
            async def gen():
                sent = {}
                base = {"id": rid, "object": "chat.completion.chunk", "created": created,
                        "model": model_name, "system_fingerprint": f"fp_{uuid.uuid4().hex[:12]}"}
                for i in range(sp.n):
                    yield sse({**base, "choices": [{"index": i, "delta": {"role": cfg.response_role},
                                                    "finish_reason": None}]})
                async for out in llm.generate(prompt, sp, request_id=rid):
                    for o in out.outputs:
                        prev = sent.get(o.index, "")
                        delta = o.text[len(prev):]
                        sent[o.index] = o.text
                        if delta or o.finish_reason is not None:
                            yield sse({**base, "choices": [{"index": o.index,
                                                            "delta": {"content": delta} if delta else {},
                                                            "finish_reason": finish(o)}]})
                    if out.finished:
                        if req.get("stream_options", {}).get("include_usage"):
                            yield sse({**base, "choices": [], "usage": usage(out)})
                        break
                yield "data: [DONE]\n\n"
            return StreamingResponse(gen(), media_type="text/event-stream")
        out = await run(prompt, None, sp, rid, request)
        if out is None:
            return err(500, "generation aborted", "server_error")
        return {
            "id": rid, "object": "chat.completion", "created": created, "model": model_name,
            "choices": [{"index": o.index,
                         "message": {"role": cfg.response_role, "content": o.text},
                         "logprobs": ({"content": [{"token": t.token, "logprob": t.logprob}
                                                   for t in o.logprobs]} if o.logprobs else None),
                         "finish_reason": finish(o)} for o in out.outputs],
            "usage": usage(out),
        }

    @app.post("/v1/completions")
    async def completions(request: Request):
        try:
            req = await request.json()
            sp = _sampling(req, 16)
            prompt, ids = prompt_of(req)
        except Exception as e:
            return err(400, f"bad request: {e}")
        rid = f"cmpl-{uuid.uuid4().hex[:24]}"
        created = int(time.time())
        if req.get("stream"):
            async def gen():
                sent = {}
                base = {"id": rid, "object": "text_completion", "created": created,
                        "model": model_name}
                async for out in llm.generate(prompt, sp, request_id=rid, prompt_token_ids=ids):
                    for o in out.outputs:
                        prev = sent.get(o.index, "")
                        delta = o.text[len(prev):]
                        sent[o.index] = o.text
                        if delta or o.finish_reason is not None:
                            yield sse({**base, "choices": [{"index": o.index, "text": delta,
                                                            "logprobs": None,
                                                            "finish_reason": finish(o)}]})
                    if out.finished:
                        break
                yield "data: [DONE]\n\n"
            return StreamingResponse(gen(), media_type="text/event-stream")
        out = await run(prompt, ids, sp, rid, request)
        if out is None:
            return err(500, "generation aborted", "server_error")
        return {
            "id": rid, "object": "text_completion", "created": created, "model": model_name,
            "choices": [{"index": o.index, "text": o.text, "logprobs": None,
                         "finish_reason": finish(o)} for o in out.outputs],
            "usage": usage(out),
        }

    return app


def serve(llm, config: Optional[ServerConfig] = None) -> None:
    import uvicorn
    cfg = config or ServerConfig()
    app = create_app(llm, cfg)
    uvicorn.run(app, host=cfg.host, port=cfg.port, ssl_keyfile=cfg.ssl_keyfile,
                ssl_certfile=cfg.ssl_certfile, log_level="warning")
