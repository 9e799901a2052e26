"""Gateway routing, eviction, auth stamping, streaming relay and metrics against mock
nodes (the reference's cortex-gateway tests use in-process mock neurons the same way)."""
import json

import httpx
import pytest
from fastapi.testclient import TestClient

from helexa_b200.gateway.app import create_gateway
from helexa_b200.gateway.core import Catalogue, CatalogueEntry, NodeState, NoRoute, Router


class MockFleet:
    def __init__(self):
        self.nodes = {
            "a": {"models": {"m1": "loaded"}, "busy": {"m1": 3}, "free": 1000},
            "b": {"models": {"m1": "loaded", "m2": "loaded"}, "busy": {"m1": 1}, "free": 500},
        }
        self.calls = []

    def handler(self, req: httpx.Request) -> httpx.Response:
        node = req.url.host.split(".")[0]
        st = self.nodes[node]
        path = req.url.path
        self.calls.append((node, req.method, path, dict(req.headers), req.content))
        if path == "/models":
            return httpx.Response(200, json={"models": [{"id": k, "status": v} for k, v in st["models"].items()]})
        if path == "/health":
            return httpx.Response(200, json={"models": {k: {"in_flight": v, "queue_depth": 0}
                                                        for k, v in st["busy"].items()}})
        if path == "/discovery":
            return httpx.Response(200, json={"devices": [{"memory_free_mb": st["free"]}]})
        if path == "/models/load":
            body = json.loads(req.content)
            st["models"][body["model_id"]] = "loaded"
            return httpx.Response(200, json={"status": "loaded"})
        if path == "/models/unload":
            st["models"].pop(json.loads(req.content)["model_id"], None)
            return httpx.Response(200, json={"status": "unloaded"})
        body = json.loads(req.content)
        if body.get("stream"):
            return httpx.Response(200, content=b'data: {"content":"x"}\n\ndata: [DONE]\n\n',
                                  headers={"content-type": "text/event-stream"})
        return httpx.Response(200, json={"model": body["model"], "served_by": node,
                                         "usage": {"completion_tokens": 2}})


def _cat():
    return Catalogue([
        CatalogueEntry("m1", "preset:x", aliases=["fast"], memory_mb=100),
        CatalogueEntry("m2", "preset:y", memory_mb=100, residency_priority=100),
        CatalogueEntry("m3", "preset:z", memory_mb=100),
    ])


def _app(fleet, **kw):
    nodes = [NodeState("a", "http://a.node"), NodeState("b", "http://b.node")]
    return create_gateway(_cat(), nodes, transport=httpx.MockTransport(fleet.handler), poll_interval_s=3600, **kw)


def test_routes_least_busy_and_rewrites_alias():
    fleet = MockFleet()
    with TestClient(_app(fleet)) as c:
        r = c.post("/v1/chat/completions", json={"model": "fast", "messages": []})
        assert r.json()["served_by"] == "b" and r.json()["model"] == "fast"
        fleet.nodes["b"]["busy"]["m1"] = 9
        c.app.state.router.observe("b", [{"id": "m1", "status": "loaded"}, {"id": "m2", "status": "loaded"}],
                                   {"models": {"m1": {"in_flight": 9}}}, 500)
        assert c.post("/v1/chat/completions", json={"model": "m1", "messages": []}).json()["served_by"] == "a"
        m = c.get("/metrics").text
        assert "cortex_requests_total" in m


def test_cold_load_evicts_lru_but_never_pinned():
    fleet = MockFleet()
    fleet.nodes["a"]["free"] = 0
    fleet.nodes["b"]["free"] = 0
    fleet.nodes["a"]["busy"]["m1"] = 0      # idle, displaceable; m2 on b is pinned
    with TestClient(_app(fleet)) as c:
        r = c.post("/v1/chat/completions", json={"model": "m3", "messages": []})
        assert r.status_code == 200
        unloads = [x for x in fleet.calls if x[2] == "/models/unload"]
        assert unloads and all(json.loads(x[4])["model_id"] != "m2" for x in unloads)
        assert any(x[2] == "/models/load" for x in fleet.calls)


def test_auth_stamps_and_strips_headers():
    fleet = MockFleet()
    with TestClient(_app(fleet, api_keys={"k1": "acct-1"}, require_auth=True)) as c:
        assert c.post("/v1/chat/completions", json={"model": "m1"}).status_code == 401
        c.post("/v1/chat/completions", json={"model": "m1"},
               headers={"authorization": "Bearer k1", "x-helexa-account": "spoofed"})
        hdr = [x for x in fleet.calls if x[2] == "/v1/chat/completions"][-1][3]
        assert hdr["x-helexa-account"] == "acct-1"


def test_streaming_relay_and_unknown_model():
    fleet = MockFleet()
    with TestClient(_app(fleet)) as c:
        r = c.post("/v1/chat/completions", json={"model": "m1", "stream": True})
        assert r.text.endswith("data: [DONE]\n\n")
        r = c.post("/v1/chat/completions", json={"model": "nope"})
        assert r.status_code == 404 and r.json()["error"]["code"] == "model_not_found"
        assert {d["id"] for d in c.get("/v1/models").json()["data"]} == {"m1", "m2", "m3"}


def test_recovering_hold_and_debounced_unhealthy():
    r = Router(_cat(), [NodeState("a", "u")])
    r.observe("a", [{"id": "m1", "status": "recovering"}], {}, 0)
    with pytest.raises(NoRoute) as e:
        r.route("m1")
    assert e.value.status == 503 and e.value.retry_after > 0
    for _ in range(3):
        r.observe("a", None, None)
    assert not r.nodes["a"].healthy


def test_entitlements_and_per_principal_metering():
    """A principal limited to m1 (reached through its alias too) is refused m2; usage is
    metered per principal into /usage and /metrics."""
    fleet = MockFleet()
    app = _app(fleet, api_keys={"k1": "acct-1", "k2": "acct-2"}, entitlements={"acct-1": {"m1"}})
    with TestClient(app) as c:
        h1, h2 = {"authorization": "Bearer k1"}, {"authorization": "Bearer k2"}
        assert c.post("/v1/chat/completions", json={"model": "m2"}, headers=h1).status_code == 403
        assert c.post("/v1/chat/completions", json={"model": "fast"}, headers=h1).status_code == 200
        assert c.post("/v1/chat/completions", json={"model": "m2"}, headers=h2).status_code == 200
        c.post("/v1/chat/completions", json={"model": "m1"})
        u = c.get("/usage").json()["principals"]
        assert u["acct-1"] == {"requests": 1, "prompt_tokens": 0, "completion_tokens": 2}
        assert u["acct-2"]["requests"] == 1 and u["anonymous"]["requests"] == 1
        m = c.get("/metrics").text
        assert 'cortex_principal_tokens_total{kind="completion",model="m1",principal="acct-1"} 2.0' in m


def test_streamed_usage_metered_from_final_usage_chunk():
    """Streamed usage comes from the usage the node reports in its final SSE event, even
    when the bytes arrive split at arbitrary points."""
    from helexa_b200.gateway.budget import SSEUsage
    body = (b'data: {"choices":[{"delta":{"content":"a"}}]}\n\n'
            b'data: {"choices":[{"delta":{"content":"\\"content\\""}}]}\n\n'
            b'data: {"choices":[],"usage":{"prompt_tokens":7,"completion_tokens":3}}\n\ndata: [DONE]\n\n')
    for cut in range(1, len(body), 5):
        u = SSEUsage()
        u.feed(body[:cut])
        u.feed(body[cut:])
        assert (u.prompt, u.completion, u.seen) == (7, 3, True)
    a = SSEUsage()
    a.feed(b'event: message_start\ndata: {"type":"message_start","message":{"usage":{"input_tokens":5,'
           b'"output_tokens":0}}}\n\nevent: message_delta\ndata: {"type":"message_delta","usage":'
           b'{"output_tokens":4}}\n\n')
    assert (a.prompt, a.completion) == (5, 4)

    fleet = MockFleet()
    orig = fleet.handler

    def handler(req):
        if req.url.path == "/v1/chat/completions" and json.loads(req.content).get("stream"):
            return httpx.Response(200, content=body, headers={"content-type": "text/event-stream"})
        return orig(req)
    nodes = [NodeState("a", "http://a.node"), NodeState("b", "http://b.node")]
    app = create_gateway(_cat(), nodes, transport=httpx.MockTransport(handler), poll_interval_s=3600,
                         api_keys={"k1": "acct-1"})
    with TestClient(app) as c:
        c.post("/v1/chat/completions", json={"model": "m1", "stream": True}, headers={"authorization": "Bearer k1"})
        u = c.get("/usage").json()["principals"]["acct-1"]
        assert (u["prompt_tokens"], u["completion_tokens"]) == (7, 3)


def test_prompt_prevalidation_against_advertised_context():
    fleet = MockFleet()
    with TestClient(_app(fleet)) as c:
        c.app.state.router.observe("a", [{"id": "m1", "status": "loaded", "limit": {"context": 100, "output": 50}}],
                                   {}, 1000)
        c.app.state.router.observe("b", [{"id": "m2", "status": "loaded"}], {}, 1000)
        n0 = len(fleet.calls)
        r = c.post("/v1/chat/completions", json={"model": "m1", "messages": [{"role": "user", "content": "x" * 2000}]})
        assert r.status_code == 400 and r.json()["error"]["code"] == "context_length_exceeded"
        assert len(fleet.calls) == n0  # refused before dispatch
        r = c.post("/v1/chat/completions", json={"model": "m1", "messages": [{"role": "user", "content": "hi"}]})
        assert r.status_code == 200


def test_budget_reserve_settle_and_rejection_codes():
    from helexa_b200.gateway.budget import BudgetExceeded, BudgetLedger, Cap
    t = [0.0]
    led = BudgetLedger({"bal": Cap(100), "win": Cap(50, window_s=60)}, clock=lambda: t[0])
    r1 = led.reserve("bal", 60)
    with pytest.raises(BudgetExceeded) as e:   # outstanding reservations count against the cap
        led.reserve("bal", 50)
    assert e.value.code == "insufficient_quota" and e.value.retry_after == 0
    led.settle(r1, 20)                          # the unused 40 come back
    led.settle(r1, 999)                         # a reservation resolves once
    assert led.snapshot("bal") == {"hard_cap": 100, "spent": 20, "reserved": 0, "window_s": 0}
    led.release(led.reserve("bal", 80))
    assert led.snapshot("bal")["reserved"] == 0
    led.settle(led.reserve("win", 50), 50)
    with pytest.raises(BudgetExceeded) as e:
        led.reserve("win", 1)
    assert e.value.code == "rate_limit_exceeded" and e.value.retry_after > 0
    t[0] = 61.0                                 # the rolling window resets
    assert led.reserve("win", 10) is not None
    assert led.reserve("nobody", 10**9) is None  # uncapped principals are not reserved

    fleet = MockFleet()
    app = _app(fleet, api_keys={"k1": "acct-1"}, budgets={"acct-1": Cap(4200)})
    with TestClient(app) as c:
        h = {"authorization": "Bearer k1"}
        # reservation = prompt estimate + max_tokens; the mock reports 2 completion tokens
        assert c.post("/v1/chat/completions", json={"model": "m1", "max_tokens": 4000}, headers=h).status_code == 200
        b = c.get("/usage").json()["principals"]["acct-1"]["budget"]
        assert b["spent"] == 2 and b["reserved"] == 0
        r = c.post("/v1/chat/completions", json={"model": "m1", "max_tokens": 5000}, headers=h)
        assert r.status_code == 429 and r.json()["error"]["code"] == "insufficient_quota"


def test_cli_gateway_config_and_status(tmp_path):
    """`helexa serve` builds the gateway from a TOML config; `helexa status` prints the
    fleet health and model placements the gateway reports."""
    from helexa_b200.cli import _gateway_from_config, status_report
    from helexa_b200.config.settings import load_settings
    p = tmp_path / "cortex.toml"
    p.write_text('[gateway]\nlisten = "127.0.0.1:31999"\npoll_interval_s = 3600\n'
                 '[[neurons]]\nname = "a"\nurl = "http://a.node/"\n'
                 '[[models]]\nmodel_id = "m1"\nsource = "preset:x"\naliases = ["fast"]\n'
                 '[auth.keys]\n"k1" = "acct-1"\n[budgets."acct-1"]\nhard_cap = 10\n')
    app = _gateway_from_config(load_settings(str(p), env={}))
    assert app.state.router.nodes["a"].url == "http://a.node"
    assert app.state.ledger.snapshot("acct-1")["hard_cap"] == 10
    replies = {"http://gw/health": {"status": "ok", "nodes": {"a": {"healthy": True, "models": ["m1"]}}},
               "http://gw/v1/models": {"data": [{"id": "m1", "loaded_on": ["a"], "limit": {"context": 4096}}]}}
    out = status_report("http://gw/", get=replies.__getitem__)
    assert "Fleet health" in out and "m1" in out and "a(loaded)" in out and "ctx=4096" in out


def test_models_listing_advertises_cost():
    cat = Catalogue([CatalogueEntry("m1", "preset:x", cost_input_per_mtok=0.2, cost_output_per_mtok=0.8)])
    fleet = MockFleet()
    app = create_gateway(cat, [NodeState("a", "http://a.node")], transport=httpx.MockTransport(fleet.handler),
                         poll_interval_s=3600)
    with TestClient(app) as c:
        d = c.get("/v1/models").json()["data"][0]
        assert d["cost"] == {"input_per_mtok": 0.2, "output_per_mtok": 0.8}


def test_browser_chat_page():
    fleet = MockFleet()
    with TestClient(_app(fleet)) as c:
        r = c.get("/ui")
        assert r.status_code == 200 and r.headers["content-type"].startswith("text/html")
        for needle in ("/v1/models", "/v1/chat/completions", "/v1/images/generations", "x-include-thinking"):
            assert needle in r.text
