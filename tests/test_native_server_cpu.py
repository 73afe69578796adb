"""The OpenAI routes on the native C++ HTTP front end, with a tiny model on
CPU: health, models, completions and chat (plain and SSE streaming), API-key
checks, CORS preflight, 404 / 400 answers, keep-alive, and abort of a
request whose client went away."""

import http.client
import json
import socket
import time

import pytest

from swiftllm_b200 import LLM
from swiftllm_b200.config import ServerConfig
from swiftllm_b200.server.native_server import NativeServer


@pytest.fixture(scope="module")
def server():
    llm = LLM("tiny-llama", load_format="dummy", device="cpu", dtype="float32", max_model_len=256)
    srv = NativeServer(llm, ServerConfig(host="127.0.0.1", port=0, api_key="sekret")).start()
    yield srv
    srv.stop()


def _req(srv, method, path, body=None, key="sekret", conn=None):
    c = conn or http.client.HTTPConnection("127.0.0.1", srv.port, timeout=60)
    h = {"Content-Type": "application/json"}
    if key:
        h["Authorization"] = f"Bearer {key}"
    c.request(method, path, body=json.dumps(body) if body is not None else None, headers=h)
    r = c.getresponse()
    return r.status, r.read(), r


def test_health_models_auth_cors(server):
    st, b, _ = _req(server, "GET", "/health", key=None)
    assert st == 200 and json.loads(b)["status"] == "ok"
    st, b, _ = _req(server, "GET", "/v1/models")
    assert st == 200 and json.loads(b)["data"][0]["id"] == "tiny-llama"
    assert _req(server, "GET", "/v1/models", key=None)[0] == 401
    assert _req(server, "GET", "/v1/models", key="wrong")[0] == 401
    assert _req(server, "GET", "/v1/models/nope")[0] == 404
    assert _req(server, "GET", "/v1/nothing")[0] == 404
    st, _, r = _req(server, "OPTIONS", "/v1/completions", key=None)
    assert st == 204 and "POST" in r.getheader("Access-Control-Allow-Methods")
    c = http.client.HTTPConnection("127.0.0.1", server.port, timeout=60)
    c.request("POST", "/v1/completions", body="{not json", headers={"Authorization": "Bearer sekret"})
    assert c.getresponse().status == 400


def test_completion_and_chat(server):
    conn = http.client.HTTPConnection("127.0.0.1", server.port, timeout=120)
    body = {"model": "tiny-llama", "prompt": [5, 6, 7, 8], "max_tokens": 7, "temperature": 0,
            "ignore_eos": True}
    st, b, _ = _req(server, "POST", "/v1/completions", body, conn=conn)
    d = json.loads(b)
    assert st == 200 and d["object"] == "text_completion" and d["usage"]["completion_tokens"] == 7
    # same connection (keep-alive), chat
    st, b, _ = _req(server, "POST", "/v1/chat/completions",
                    {"messages": [{"role": "user", "content": "hi"}], "max_tokens": 5,
                     "temperature": 0, "ignore_eos": True}, conn=conn)
    d = json.loads(b)
    assert st == 200 and d["choices"][0]["message"]["role"] == "assistant"
    assert d["usage"]["completion_tokens"] == 5
    m = json.loads(_req(server, "GET", "/metrics")[1])
    assert m["scheduler"]["completed_requests"] >= 2 and m["http"]["requests"] >= 3


def test_streaming_matches_plain(server):
    body = {"prompt": [9, 10, 11], "max_tokens": 6, "temperature": 0, "ignore_eos": True}
    plain = json.loads(_req(server, "POST", "/v1/completions", body)[1])["choices"][0]["text"]
    st, b, r = _req(server, "POST", "/v1/completions", {**body, "stream": True})
    assert st == 200 and r.getheader("Content-Type") == "text/event-stream"
    events = [ln[6:] for ln in b.decode().split("\n") if ln.startswith("data: ")]
    assert events[-1] == "[DONE]"
    chunks = [json.loads(e) for e in events[:-1]]
    assert "".join(c["choices"][0]["text"] for c in chunks) == plain
    assert chunks[-1]["choices"][0]["finish_reason"] == "length"
    st, b, _ = _req(server, "POST", "/v1/chat/completions",
                    {"messages": [{"role": "user", "content": "x"}], "max_tokens": 4, "stream": True,
                     "temperature": 0, "ignore_eos": True, "stream_options": {"include_usage": True}})
    events = [ln[6:] for ln in b.decode().split("\n") if ln.startswith("data: ")]
    objs = [json.loads(e) for e in events[:-1]]
    assert objs[0]["choices"][0]["delta"]["role"] == "assistant"
    assert objs[-1]["usage"]["completion_tokens"] == 4


def test_disconnect_aborts(server):
    s = socket.create_connection(("127.0.0.1", server.port))
    body = json.dumps({"prompt": [1, 2, 3], "max_tokens": 200, "stream": True, "ignore_eos": True})
    s.sendall(("POST /v1/completions HTTP/1.1\r\nHost: x\r\nAuthorization: Bearer sekret\r\n"
               f"Content-Length: {len(body)}\r\n\r\n{body}").encode())
    s.recv(100)
    s.close()
    for _ in range(200):
        if not server.active:
            break
        time.sleep(0.05)
    assert not server.active
    assert _req(server, "GET", "/health", key=None)[0] == 200
