"""OpenAI-compatible server on the CPU runner (tiny LLaMA, byte tokenizer):
routes, streaming SSE, usage counts, finish reasons, API-key check, metrics.
Parity: crates/swiftllm-server/src/lib.rs:46-94, api/openai.rs."""

import json

import pytest

fastapi = pytest.importorskip("fastapi")
from fastapi.testclient import TestClient  # noqa: E402

from swiftllm_b200 import AsyncLLM, ServerConfig  # noqa: E402
from swiftllm_b200.server.openai_server import create_app  # noqa: E402


@pytest.fixture(scope="module")
def client():
    llm = AsyncLLM("tiny-llama", load_format="dummy", device="cpu", dtype="float32",
                   max_num_seqs=8, max_model_len=512)
    app = create_app(llm, ServerConfig(api_key="sekret", served_model_name="tiny"))
    with TestClient(app) as c:
        c.headers.update({"Authorization": "Bearer sekret"})
        yield c
    llm.shutdown()


def test_health_models_and_auth(client):
    assert client.get("/health").json()["status"] == "ok"
    assert client.get("/v1/models").json()["data"][0]["id"] == "tiny"
    assert client.get("/v1/models/tiny").status_code == 200
    assert client.get("/v1/models/nope").status_code == 404
    r = client.post("/v1/completions", json={"prompt": "x"}, headers={"Authorization": "Bearer no"})
    assert r.status_code == 401


def test_completion_non_stream(client):
    r = client.post("/v1/completions", json={"model": "tiny", "prompt": "Hello", "max_tokens": 5,
                                             "temperature": 0, "ignore_eos": True})
    d = r.json()
    assert r.status_code == 200 and d["object"] == "text_completion" and d["id"].startswith("cmpl-")
    assert d["choices"][0]["finish_reason"] == "length"
    assert d["usage"]["completion_tokens"] == 5 and d["usage"]["prompt_tokens"] == 6


def test_chat_non_stream_and_n(client):
    r = client.post("/v1/chat/completions", json={
        "model": "tiny", "messages": [{"role": "user", "content": "hi"}], "max_tokens": 4,
        "n": 2, "temperature": 0.8, "seed": 1, "ignore_eos": True})
    d = r.json()
    assert d["object"] == "chat.completion" and d["id"].startswith("chatcmpl-")
    assert len(d["choices"]) == 2 and d["choices"][0]["message"]["role"] == "assistant"
    assert d["usage"]["completion_tokens"] == 8


def test_chat_stream(client):
    with client.stream("POST", "/v1/chat/completions", json={
            "model": "tiny", "messages": [{"role": "user", "content": "hi"}], "max_tokens": 6,
            "stream": True, "temperature": 0, "ignore_eos": True}) as r:
        lines = [ln for ln in r.iter_lines() if ln.startswith("data: ")]
    assert lines[-1] == "data: [DONE]"
    chunks = [json.loads(ln[6:]) for ln in lines[:-1]]
    assert chunks[0]["choices"][0]["delta"]["role"] == "assistant"
    assert chunks[-1]["choices"][0]["finish_reason"] == "length"
    assert all(c["object"] == "chat.completion.chunk" for c in chunks)


def test_completion_stream_and_metrics(client):
    with client.stream("POST", "/v1/completions", json={
            "prompt": [1, 2, 3], "max_tokens": 3, "stream": True, "temperature": 0,
            "ignore_eos": True}) as r:
        lines = [ln for ln in r.iter_lines() if ln.startswith("data: ")]
    assert lines[-1] == "data: [DONE]" and len(lines) >= 2
    m = client.get("/metrics").json()
    assert set(m) == {"scheduler", "memory", "execution"}


def test_bad_request(client):
    assert client.post("/v1/chat/completions", json={"model": "tiny"}).status_code == 400
