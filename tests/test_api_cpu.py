"""HTTP API on a CPU-served tiny model: node endpoints, OpenAI chat / completions /
responses, Anthropic messages, SSE framing, error envelopes and admission refusals
(the reference's tests/api.rs coverage)."""
import json

import pytest
from fastapi.testclient import TestClient

from helexa_b200.server.app import create_app


@pytest.fixture(scope="module")
def client():
    app = create_app()
    with TestClient(app) as c:
        r = c.post("/models/load", json={"model_id": "tiny", "source": "preset:tiny-qwen3-next", "device": "cpu",
                                         "max_batch": 2, "max_len": 512, "max_queue_depth": 1, "max_wait_s": 0.5})
        assert r.status_code == 200, r.text
        yield c


def _sse(text):
    out = []
    for block in text.split("\n\n"):
        for line in block.splitlines():
            if line.startswith("data: "):
                out.append(line[6:])
    return out


def test_node_endpoints(client):
    assert client.get("/version").json()["name"] == "helexa-b200"
    assert "devices" in client.get("/discovery").json()
    h = client.get("/health").json()
    assert h["status"] == "ok" and "tiny" in h["models"]
    ms = client.get("/models").json()["models"]
    assert ms[0]["id"] == "tiny" and ms[0]["status"] == "loaded" and ms[0]["limit"]["context"] == 512
    assert client.get("/v1/models").json()["data"][0]["id"] == "tiny"
    assert client.get("/models/tiny/capabilities").json()["tool_call"] is True
    assert client.get("/models/nope/endpoint").status_code == 404


def test_chat_completion_nonstream_and_stream(client):
    body = {"model": "tiny", "messages": [{"role": "user", "content": "hi"}], "max_tokens": 5, "temperature": 0}
    r = client.post("/v1/chat/completions", json=body)
    assert r.status_code == 200, r.text
    j = r.json()
    assert j["object"] == "chat.completion" and j["usage"]["completion_tokens"] <= 5
    assert "helexa_timing" in j["usage"]
    body["stream"] = True
    r = client.post("/v1/chat/completions", json=body)
    chunks = _sse(r.text)
    assert chunks[-1] == "[DONE]"
    first = json.loads(chunks[0])
    assert first["choices"][0]["delta"]["role"] == "assistant"
    last = json.loads(chunks[-2])
    assert last["choices"][0]["finish_reason"] in ("length", "stop") and "usage" in last


def test_completions_responses_anthropic(client):
    r = client.post("/v1/completions", json={"model": "tiny", "prompt": "abc", "max_tokens": 3, "temperature": 0})
    assert r.json()["object"] == "text_completion"
    r = client.post("/v1/responses", json={"model": "tiny", "input": "hello", "max_output_tokens": 3})
    assert r.json()["object"] == "response" and r.json()["status"] == "completed"
    r = client.post("/v1/responses", json={"model": "tiny", "input": "x", "previous_response_id": "resp_1"})
    assert r.status_code == 400 and r.json()["error"]["code"] == "unsupported_parameter"
    r = client.post("/v1/responses", json={"model": "tiny", "input": "hello", "max_output_tokens": 3,
                                           "stream": True})
    assert "event: response.completed" in r.text
    r = client.post("/v1/messages", json={"model": "tiny", "max_tokens": 4, "system": "be brief",
                                          "messages": [{"role": "user", "content": "hi"}]})
    j = r.json()
    assert j["type"] == "message" and j["stop_reason"] in ("max_tokens", "end_turn")
    r = client.post("/v1/messages", json={"model": "tiny", "max_tokens": 4, "stream": True,
                                          "messages": [{"role": "user", "content": [{"type": "text", "text": "x"}]}]})
    assert "event: message_start" in r.text and "event: message_stop" in r.text


def test_errors(client):
    r = client.post("/v1/chat/completions", json={"model": "missing", "messages": [{"role": "user", "content": "x"}]})
    assert r.status_code == 404 and r.json()["error"]["code"] == "model_not_found"
    r = client.post("/v1/images/generations", json={"model": "tiny", "prompt": "cat"})
    assert r.status_code == 400 and r.json()["error"]["code"] == "wrong_modality"
    r = client.post("/v1/chat/completions", json={"model": "tiny", "messages": []})
    assert r.status_code == 400
    r = client.post("/models/unload", json={"model_id": "nope"})
    assert r.status_code == 404


def test_refuses_below_free_memory_floor(client):
    """Below the free-device-memory floor new requests get 503 insufficient_vram."""
    sm = client.app.state.registry.models["tiny"]
    old = sm.free_vram_mb
    try:
        sm.free_vram_mb = lambda: sm.min_free_vram_mb - 1
        r = client.post("/v1/chat/completions", json={"model": "tiny", "max_tokens": 2,
                                                      "messages": [{"role": "user", "content": "hi"}]})
        assert r.status_code == 503 and r.json()["error"]["code"] == "insufficient_vram", r.text
    finally:
        sm.free_vram_mb = old
    r = client.post("/v1/chat/completions", json={"model": "tiny", "max_tokens": 2,
                                                  "messages": [{"role": "user", "content": "hi"}]})
    assert r.status_code == 200
