"""OpenAI-compatible server on the native HTTP front end.

The C++ front end (csrc/core/http_server.cpp) owns the sockets: it parses
HTTP/1.1, answers CORS preflight, /health and API-key rejections itself, and
queues every other request. This module runs ONE Python thread that alternates
between taking queued requests (``HttpServer.poll``) and stepping the engine
(``LLMEngine.step``); streamed deltas leave as SSE chunks, complete answers as
one response. There is no asyncio loop and no per-request coroutine between
the engine and the socket. A request whose client disconnects is aborted.

Same routes, JSON shapes and defaults as server/openai_server.py (the FastAPI
variant, kept for deployments that want ASGI middleware).

Parity: crates/swiftllm-server/src/lib.rs:27-126 (router, /health, /metrics),
crates/swiftllm-server/src/api/openai.rs:25-320 (schemas),
crates/swiftllm-server/src/streaming.rs:7-28 (SSE).
"""

from __future__ import annotations

import json
import threading
import time
import uuid
from dataclasses import dataclass, field
from typing import Any, Dict, Optional

from .. import _core
from ..config import ServerConfig
from ..engine.tokenizer import chat_prompt
from ..utils.logging import get_logger
from .openai_server import VERSION, _sampling

log = get_logger(__name__)


@dataclass
class _Active:
    conn: int
    kind: str            # "chat" | "completion"
    stream: bool
    created: int
    include_usage: bool = False
    sent: Dict[int, str] = field(default_factory=dict)


def _err(status: int, msg: str, kind: str = "invalid_request_error") -> str:
    return json.dumps({"error": {"message": msg, "type": kind, "code": status}})


class NativeServer:
    def __init__(self, llm, config: Optional[ServerConfig] = None):
        self.cfg = config or ServerConfig()
        self.llm = llm
        self.engine = llm.llm_engine
        self.engine._ensure_initialized()
        self.model_name = self.cfg.served_model_name or self.engine.config.model
        self.http = _core.HttpServer(self.cfg.host, int(self.cfg.port), self.cfg.api_key or "")
        self.port = self.http.port
        self.active: Dict[str, _Active] = {}
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None

    # ------------------------------------------------------------ lifecycle
    def start(self) -> "NativeServer":
        self.http.start()
        self._thread = threading.Thread(target=self.serve_forever, name="swiftllm-native-server",
                                        daemon=True)
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=30)
        self.http.stop()

    def serve_forever(self) -> None:
        self.http.start()
        log.info("native OpenAI server on %s:%d", self.cfg.host, self.port)
        while not self._stop.is_set():
            busy = self.engine.has_unfinished_requests()
            r = self.http.poll(0.0 if busy else 0.05)
            while r is not None:
                try:
                    self._handle(*r)
                except Exception as e:  # a handler bug must not stop the server
                    log.exception("request failed")
                    self.http.respond(r[0], 500, "application/json", _err(500, str(e), "server_error"))
                r = self.http.poll(0.0)
            for rid, st in list(self.active.items()):
                if not self.http.is_open(st.conn):
                    self.engine.abort_request(rid)
                    self.active.pop(rid, None)
            if self.engine.has_unfinished_requests():
                for out in self.engine.step():
                    self._emit(out)

    # ------------------------------------------------------------ requests
    def _json(self, conn: int, obj: Any, status: int = 200) -> None:
        self.http.respond(conn, status, "application/json", json.dumps(obj))

    def _model_card(self) -> Dict[str, Any]:
        return {"id": self.model_name, "object": "model", "created": int(time.time()),
                "owned_by": "swiftllm"}

    def _handle(self, conn: int, method: str, target: str, body: bytes) -> None:
        path = target.split("?", 1)[0]
        if method == "GET" and path == "/v1/models":
            return self._json(conn, {"object": "list", "data": [self._model_card()]})
        if method == "GET" and path.startswith("/v1/models/"):
            mid = path[len("/v1/models/"):]
            if mid != self.model_name:
                return self.http.respond(conn, 404, "application/json",
                                         _err(404, f"model {mid!r} not found", "not_found_error"))
            return self._json(conn, self._model_card())
        if method == "GET" and path == "/metrics":
            return self._json(conn, self._metrics())
        if method == "POST" and path in ("/v1/chat/completions", "/v1/completions"):
            return self._generate(conn, path.endswith("chat/completions"), body)
        self.http.respond(conn, 404, "application/json",
                          _err(404, f"no route {method} {path}", "not_found_error"))

    def _metrics(self) -> Dict[str, Any]:
        s = self.engine.stats()
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
            "http": self.http.stats(),
        }

    def _generate(self, conn: int, chat: bool, body: bytes) -> None:
        try:
            req = json.loads(body or b"{}")
            sp = _sampling(req, 256 if chat else 16)
            ids = None
            if chat:
                msgs = req["messages"]
                tok = self.engine.tokenizer
                if hasattr(tok, "apply_chat_template") and getattr(tok, "chat_template", None):
                    prompt = tok.apply_chat_template(msgs, add_generation_prompt=True, tokenize=False)
                else:
                    prompt = chat_prompt(msgs)
            else:
                prompt = req.get("prompt", "")
                if isinstance(prompt, list):
                    if prompt and isinstance(prompt[0], int):
                        prompt, ids = None, prompt
                    else:
                        prompt = prompt[0] if prompt else ""
            rid = f"{'chatcmpl' if chat else 'cmpl'}-{uuid.uuid4().hex[:24]}"
            stream = bool(req.get("stream"))
            self.engine.add_request(rid, prompt=prompt, sampling_params=sp, prompt_token_ids=ids,
                                    stream=stream)
        except Exception as e:
            return self.http.respond(conn, 400, "application/json", _err(400, f"bad request: {e}"))
        st = _Active(conn, "chat" if chat else "completion", stream, int(time.time()),
                     bool((req.get("stream_options") or {}).get("include_usage")))
        self.active[rid] = st
        if stream:
            self.http.stream_start(conn)
            if chat:
                base = self._base(rid, st)
                for i in range(sp.n):
                    self._sse(conn, {**base, "choices": [{"index": i, "delta": {"role": self.cfg.response_role},
                                                          "finish_reason": None}]})

    # ------------------------------------------------------------ outputs
    def _base(self, rid: str, st: _Active) -> Dict[str, Any]:
        return {"id": rid, "object": "chat.completion.chunk" if st.kind == "chat" else "text_completion",
                "created": st.created, "model": self.model_name}

    def _sse(self, conn: int, obj: Any) -> None:
        self.http.stream_send(conn, f"data: {json.dumps(obj)}\n\n")

    @staticmethod
    def _usage(out) -> Dict[str, int]:
        p = len(out.prompt_token_ids)
        c = sum(len(o.token_ids) for o in out.outputs)
        return {"prompt_tokens": p, "completion_tokens": c, "total_tokens": p + c}

    @staticmethod
    def _finish(o) -> Optional[str]:
        return o.finish_reason.value if o.finish_reason is not None else None

    def _emit(self, out) -> None:
        st = self.active.get(out.request_id)
        if st is None:
            return
        if st.stream:
            base = self._base(out.request_id, st)
            for o in out.outputs:
                prev = st.sent.get(o.index, "")
                delta = o.text[len(prev):]
                st.sent[o.index] = o.text
                if delta or o.finish_reason is not None:
                    if st.kind == "chat":
                        ch = {"index": o.index, "delta": {"content": delta} if delta else {},
                              "finish_reason": self._finish(o)}
                    else:
                        ch = {"index": o.index, "text": delta, "logprobs": None,
                              "finish_reason": self._finish(o)}
                    self._sse(st.conn, {**base, "choices": [ch]})
            if out.finished:
                if st.include_usage:
                    self._sse(st.conn, {**base, "choices": [], "usage": self._usage(out)})
                self.http.stream_send(st.conn, "data: [DONE]\n\n")
                self.http.stream_end(st.conn)
                self.active.pop(out.request_id, None)
            return
        if not out.finished:
            return
        self.active.pop(out.request_id, None)
        if st.kind == "chat":
            choices = [{"index": o.index, "message": {"role": self.cfg.response_role, "content": o.text},
                        "logprobs": ({"content": [{"token": t.token, "logprob": t.logprob}
                                                  for t in o.logprobs]} if o.logprobs else None),
                        "finish_reason": self._finish(o)} for o in out.outputs]
            obj = "chat.completion"
        else:
            choices = [{"index": o.index, "text": o.text, "logprobs": None,
                        "finish_reason": self._finish(o)} for o in out.outputs]
            obj = "text_completion"
        self._json(st.conn, {"id": out.request_id, "object": obj, "created": st.created,
                             "model": self.model_name, "choices": choices, "usage": self._usage(out)})


def serve_native(llm, config: Optional[ServerConfig] = None) -> None:
    """Blocking: serve until interrupted."""
    srv = NativeServer(llm, config)
    try:
        srv.serve_forever()
    except KeyboardInterrupt:
        pass
    finally:
        srv.http.stop()
