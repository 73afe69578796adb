// Native HTTP/1.1 front end for the OpenAI-compatible server.
//
// One I/O thread runs an epoll loop: it accepts connections, parses requests
// (request line, headers, Content-Length bodies; keep-alive), answers the
// cheap routes itself (CORS preflight, /health, missing or wrong Bearer key
// on /v1/*) and hands every other request to the engine side through a
// queue. The engine side (Python, one thread, no asyncio) pulls requests with
// poll(), and answers with respond() or with a chunked Server-Sent-Events
// stream (stream_start / stream_send / stream_end). Responses are queued to
// the I/O thread, which owns every socket write (non-blocking, buffered,
// woken through an eventfd). A client that disconnects is reported by
// is_open() so the engine can abort its request.
//
// Parity: crates/swiftllm-server/src/lib.rs:27-126 (axum router: CORS for any
// origin, /health, /metrics, OpenAI routes; the api key is stored but never
// checked there) and crates/swiftllm-server/src/streaming.rs:7-28 (SSE).
#pragma once
#include <pybind11/pybind11.h>

void bind_http_server(pybind11::module_& m);
