"""Tensor-parallel serving through the node API on CPU: `POST /models/load` with
`tensor_parallel: 2` spawns two gloo rank processes (each a full fp32 reference
model), requests run through the rank-0 leader in lockstep, a rank failure poisons the
model, and the next request triggers recovery (unload = rank processes stopped, reload
from the retained spec). Mirrors the reference's host-only TP worker lifecycle tests."""
import time

import pytest
from fastapi.testclient import TestClient

from helexa_b200.server.app import create_app

BODY = {"messages": [{"role": "user", "content": "count to three"}], "max_tokens": 6, "temperature": 0}


def _load(c, mid, tp, **kw):
    spec = {"model_id": mid, "source": "preset:tiny-qwen3-next", "device": "cpu", "tensor_parallel": tp,
            "max_batch": 2, "max_len": 512}
    spec.update(kw)
    r = c.post("/models/load", json=spec)
    assert r.status_code == 200, r.text


def _chat(c, mid):
    r = c.post("/v1/chat/completions", json=dict(BODY, model=mid))
    return r.status_code, r.json()


@pytest.mark.timeout(600)
def test_tp2_load_chat_unload_matches_tp1():
    with TestClient(create_app()) as c:
        _load(c, "tp1", 1)
        _load(c, "tp2", 2)
        ms = {m["id"]: m for m in c.get("/models").json()["models"]}
        assert ms["tp2"]["tensor_parallel"] == 2 and ms["tp2"]["status"] == "loaded"
        s1, j1 = _chat(c, "tp1")
        s2, j2 = _chat(c, "tp2")
        assert s1 == s2 == 200
        assert j2["choices"][0]["message"]["content"] == j1["choices"][0]["message"]["content"]
        # a second identical request hits the prefix snapshot held by both ranks
        s3, j3 = _chat(c, "tp2")
        assert s3 == 200 and j3["choices"][0]["message"]["content"] == j1["choices"][0]["message"]["content"]
        reg = c.app.state.registry
        procs = reg.models["tp2"].engine.runner.procs
        assert c.post("/models/unload", json={"model_id": "tp2"}).status_code == 200
        assert all(p.poll() is not None for p in procs)  # every rank process stopped


@pytest.mark.timeout(600)
def test_tp2_rank_failure_poisons_then_recovers(monkeypatch):
    with TestClient(create_app()) as c:
        _load(c, "ok", 1)
        s, j = _chat(c, "ok")
        assert s == 200
        # rank 1 raises on a prefill of exactly this prompt's length
        n = j["usage"]["prompt_tokens"]
        monkeypatch.setenv("HELEXA_DEBUG_TP_FAIL", f"1:{n}")
        _load(c, "tp", 2, prefix_cache_mb=0)
        s, j = _chat(c, "tp")
        assert s != 200 or j["choices"][0]["finish_reason"] == "error"
        reg = c.app.state.registry
        old_procs = reg.models["tp"].engine.runner.procs
        assert reg.models["tp"].status == "poisoned"
        monkeypatch.delenv("HELEXA_DEBUG_TP_FAIL")
        s, j = _chat(c, "tp")  # triggers recovery
        assert s == 503 and j["error"]["code"] == "model_recovering"
        for _ in range(600):
            m = reg.models.get("tp")
            if m is not None and m.status == "loaded" and "tp" not in reg.recovering:
                break
            time.sleep(0.5)
        assert all(p.poll() is not None for p in old_procs)
        s, j = _chat(c, "tp")
        assert s == 200 and j["choices"][0]["finish_reason"] in ("length", "stop")
