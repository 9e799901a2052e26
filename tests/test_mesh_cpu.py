"""Federation router and tools service (the reference's helexa-router and helexa-tools
tests: selection order, failover, alias rewrite, catalogue merge, SSRF rules,
redirect re-checks, content-type gates, extraction and truncation)."""
import json
import socket

import httpx
import pytest
from fastapi.testclient import TestClient

from helexa_b200.mesh import router as rt
from helexa_b200.mesh import tools


def _entry(mid, loaded, feasible=(), ctx=4096, cost=None, caps=("text",)):
    e = {"id": mid, "object": "model", "loaded": loaded, "feasible_on": list(feasible), "limit": {"context": ctx},
         "capabilities": list(caps)}
    if cost:
        e["cost"] = cost
    return e


def _cortex_transport(state):
    """Mock cortexes a (loaded m1) and b (feasible m1, loaded m2); state['down'] lists
    cortexes whose connections fail."""
    def handler(req: httpx.Request):
        host = req.url.host
        if host in state["down"]:
            raise httpx.ConnectError("down", request=req)
        if req.url.path == "/v1/models":
            data = {"a": [_entry("m1", True, ctx=8192, cost={"input_per_mtok": 2, "output_per_mtok": 2})],
                    "b": [_entry("m1", False, ["n1"], ctx=4096, cost={"input_per_mtok": 1, "output_per_mtok": 1},
                                 caps=("text", "vision")),
                          _entry("m2", True)]}[host]
            return httpx.Response(200, json={"data": data})
        if req.url.path == "/health":
            return httpx.Response(200, json={"nodes": {"healthy": {"a": 1, "b": 3}[host], "total": 3}})
        body = json.loads(req.content)
        state["hits"].append((host, req.url.path, body["model"]))
        return httpx.Response(200, json={"served_by": host, "model": body["model"]})
    return httpx.MockTransport(handler)


def _router(state, region=None):
    cfg = rt.RouterConfig(cortexes=[rt.CortexEndpoint("a", "http://a", "eu"), rt.CortexEndpoint("b", "http://b", "us")],
                          aliases={"fast": "m2"}, region=region)
    return rt.create_router(cfg, transport=_cortex_transport(state), poll=False)


def test_router_selection_failover_alias_and_catalogue():
    state = {"down": set(), "hits": []}
    app = _router(state)
    with TestClient(app) as c:
        c.portal.call(app.state.poll_once)
        # loaded beats feasible even with fewer healthy nodes
        r = c.post("/v1/chat/completions", json={"model": "m1", "messages": []})
        assert r.status_code == 200 and r.json()["served_by"] == "a"
        # alias rewrite
        r = c.post("/v1/chat/completions", json={"model": "fast", "messages": []})
        assert r.json() == {"served_by": "b", "model": "m2"}
        # failover when the preferred cortex refuses connections
        state["down"].add("a")
        r = c.post("/v1/messages", json={"model": "m1", "messages": []})
        assert r.json()["served_by"] == "b"
        state["down"].clear()
        assert c.post("/v1/chat/completions", json={"model": "nope"}).status_code == 404
        assert c.post("/v1/chat/completions", content=b"{}").json()["error"]["code"] == "missing_model_field"
        models = {m["id"]: m for m in c.get("/v1/models").json()["data"]}
        m1 = models["m1"]
        assert m1["loaded"] and m1["feasible_on"] == ["a", "b"] and m1["limit"]["context"] == 4096
        assert m1["cost"]["input_per_mtok"] == 1 and set(m1["capabilities"]) == {"text", "vision"}
        assert m1["locations"] == [{"node": "a", "status": "loaded"}]
        assert c.get("/health").json()["cortexes"] == {"configured": 2, "reachable": 2}


def test_router_unreachable_after_three_failed_polls():
    st = rt.RouterState(rt.RouterConfig(cortexes=[rt.CortexEndpoint("a", "http://a")]))
    st.observe("a", [_entry("m1", True)], 1)
    assert st.select("m1")[0] == "candidates"
    for i in range(3):
        st.observe("a", None)
        assert st.topology["a"].reachable == (i < 2)
    assert st.select("m1") == ("unreachable", None)
    assert st.select("zzz") == ("unknown", None)


def test_router_region_and_health_ranking():
    cfg = rt.RouterConfig(cortexes=[rt.CortexEndpoint("x", "http://x", "us"), rt.CortexEndpoint("y", "http://y", "eu"),
                                    rt.CortexEndpoint("z", "http://z", "eu")], region="eu")
    st = rt.RouterState(cfg)
    for n, h in (("x", 9), ("y", 1), ("z", 2)):
        st.observe(n, [_entry("m", True)], h)
    assert [e.name for e in st.select("m")[1]] == ["z", "y", "x"]


def test_ssrf_rules():
    ok = ["https://example.com/page", "http://sub.example.co.uk/x?y=1", "https://93.184.216.34/"]
    for u in ok:
        tools.check_url(u)
    bad = ["ftp://example.com/", "file:///etc/passwd", "http://localhost/", "http://intranet/",
           "http://build.corp.internal:8090/", "http://printer.local/", "http://nas.lan/", "http://x.home.arpa/",
           "http://127.0.0.1/", "http://10.1.2.3/", "http://172.16.0.1/", "http://192.168.1.1/", "http://169.254.169.254/",
           "http://100.64.0.1/", "http://0.0.0.0/", "http://198.18.0.1/", "http://224.0.0.1/", "http://[::1]/",
           "http://[fd00::1]/", "http://[fe80::1]/", "http://[::ffff:127.0.0.1]/", "http://[2001:db8::1]/"]
    for u in bad:
        with pytest.raises(tools.Denied):
            tools.check_url(u)
    assert tools.ip_allowed("2606:4700::1111")

    def resolver(host, port, type=0):
        return {"good.example": [(0, 0, 0, "", ("93.184.216.34", port))],
                "rebind.example": [(0, 0, 0, "", ("93.184.216.34", port)), (0, 0, 0, "", ("10.0.0.5", port))]}[host]
    assert tools.resolve_validated("good.example", 80, resolver) == "93.184.216.34"
    with pytest.raises(tools.Denied):
        tools.resolve_validated("rebind.example", 80, resolver)


def _fake_resolver(host, port, type=0):
    table = {"site.example": "93.184.216.34", "evil.example": "10.0.0.9"}
    if host not in table:
        raise socket.gaierror("nx")
    return [(0, 0, 0, "", (table[host], port))]


def _site_transport():
    page = ("<html><head><title> The Title </title><script>var x=1</script></head><body><nav>menu</nav>"
            "<article><h1>Heading</h1><p>First   para.</p><p>Second &amp; last.</p></article><footer>f</footer>"
            "</body></html>")

    def handler(req: httpx.Request):
        assert req.url.host == "93.184.216.34" and req.headers["host"].startswith("site.example")
        p = req.url.path
        if p == "/page":
            return httpx.Response(200, text=page, headers={"content-type": "text/html; charset=utf-8"})
        if p == "/plain":
            return httpx.Response(200, text="x" * 50, headers={"content-type": "text/plain"})
        if p == "/pdf":
            return httpx.Response(200, content=b"%PDF", headers={"content-type": "application/pdf"})
        if p == "/hop":
            return httpx.Response(302, headers={"location": "/page"})
        if p == "/to-internal":
            return httpx.Response(302, headers={"location": "http://evil.example/"})
        if p == "/loop":
            return httpx.Response(302, headers={"location": "/loop"})
        return httpx.Response(404)
    return httpx.MockTransport(handler)


def test_tools_fetch_service():
    app = tools.create_tools_app(tools.ToolsConfig(max_text_chars=20), transport=_site_transport(),
                                 resolver=_fake_resolver)
    with TestClient(app) as c:
        assert c.get("/health").json()["status"] == "ok"
        j = c.get("/fetch", params={"url": "http://site.example/page"}).json()
        assert j["title"] == "The Title" and j["text"].startswith("Heading\nFirst para.") and j["truncated"]
        assert "menu" not in j["text"] and "var x" not in j["text"]
        j = c.get("/fetch", params={"url": "http://site.example/hop"}).json()
        assert j["url"] == "http://site.example/page"
        j = c.get("/fetch", params={"url": "http://site.example/plain"}).json()
        assert j["text"] == "x" * 20 and j["truncated"] and j["title"] == ""
        assert c.get("/fetch", params={"url": "http://site.example/pdf"}).status_code == 415
        assert c.get("/fetch", params={"url": "http://site.example/to-internal"}).status_code == 400
        assert c.get("/fetch", params={"url": "http://site.example/loop"}).status_code == 502
        assert c.get("/fetch", params={"url": "http://site.example/missing"}).status_code == 502
        assert c.get("/fetch", params={"url": "http://127.0.0.1/"}).status_code == 400
        assert c.get("/fetch", params={"url": "http://nx.example/"}).status_code == 400
    full = tools.extract_readable("<p>a</p><p>b</p>")
    assert full == ("", "a\nb")


# ---- upstream ledger ------------------------------------------------------------
from helexa_b200.mesh import upstream as up  # noqa: E402


def test_ledger_reserve_settle_release_no_overshoot():
    L = up.Ledger()
    aid = L.create_account("a@x.io", allocation=1000)
    k1, raw1 = L.create_key(aid, "all")
    k2, _ = L.create_key(aid, "capped", "hardcap", 300)
    k3, _ = L.create_key(aid, "half", "percent", 50)
    assert L.resolve_key(raw1)["hard_cap"] == 1000 and L.resolve_key("nope") is None
    r = L.reserve(aid, k2, 300)
    with pytest.raises(up.InsufficientQuota) as e:
        L.reserve(aid, k2, 1)
    assert e.value.available == 0
    L.settle(r, 120)                    # charge 120, return 180
    assert L.snapshot(aid, k2) == {"hard_cap": 300, "spent": 120, "reserved": 0}
    L.settle(r, 999)                    # idempotent
    assert L.account(aid)["allocation_spent"] == 120
    r = L.reserve(aid, k3, 500)
    L.settle(r, 10_000)                 # capped at the reservation
    assert L.snapshot(aid, k3)["spent"] == 500
    # account-level availability now 1000 - 620 = 380 even for the 100% key
    with pytest.raises(up.InsufficientQuota) as e:
        L.reserve(aid, k1, 381)
    assert e.value.available == 380
    r = L.reserve(aid, k1, 380)
    L.release(r)
    assert L.account(aid)["allocation_reserved"] == 0 and L.account(aid)["allocation_spent"] == 620
    r = L.reserve(aid, k1, 10)
    L.db.execute("UPDATE reservations SET created_at = created_at - 10000 WHERE id = ?", (r,))
    assert L.sweep_stale(60) == 1 and L.account(aid)["allocation_reserved"] == 0
    assert L.archive_key(aid, k1) and L.resolve_key(raw1) is None
    code = L.mint_code(5000)
    assert L.redeem(aid, code) == 5000
    with pytest.raises(up.LedgerError):
        L.redeem(aid, code)


def test_ledger_concurrent_reservations_never_overshoot():
    import threading
    L = up.Ledger()
    aid = L.create_account(allocation=1000)
    kid, _ = L.create_key(aid)
    ok = []

    def worker():
        for _ in range(20):
            try:
                ok.append(L.reserve(aid, kid, 7))
            except up.InsufficientQuota:
                pass

    ts = [threading.Thread(target=worker) for _ in range(8)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert len(ok) == 1000 // 7 and L.account(aid)["allocation_reserved"] == 7 * len(ok)


def test_upstream_http_surface():
    app = up.create_upstream(up.UpstreamConfig(operator_tokens={"op-secret": "op1"}, signup_allocation=100))
    with TestClient(app) as c:
        r = c.post("/web/v1/register", json={"email": "u@x.io", "password": "correct horse"})
        sess = {"Authorization": "Bearer " + r.json()["session"]}
        assert c.post("/web/v1/register", json={"email": "u@x.io", "password": "correct horse"}).status_code == 409
        assert c.post("/web/v1/login", json={"email": "u@x.io", "password": "wrong pass"}).status_code == 401
        assert c.post("/web/v1/login", json={"email": "u@x.io", "password": "correct horse"}).status_code == 200
        key = c.post("/web/v1/keys", json={"label": "cli", "limit_kind": "hardcap", "limit_value": 60},
                     headers=sess).json()
        assert c.get("/web/v1/allocation", headers=sess).json()["available"] == 100
        op = {"Authorization": "Bearer op-secret"}
        assert c.post("/authz/v1/resolve", json={"api_key": key["key"]}).status_code == 401
        res = c.post("/authz/v1/resolve", json={"api_key": key["key"]}, headers=op).json()
        p = res["principal"]
        assert res["snapshot"]["hard_cap"] == 60
        rid = c.post("/authz/v1/reserve", json={**p, "max_tokens": 50}, headers=op).json()["reservation_id"]
        rej = c.post("/authz/v1/reserve", json={**p, "max_tokens": 20}, headers=op).json()
        assert rej == {"rejected": {"kind": "insufficient_quota", "requested": 20, "available": 10}}
        c.post("/authz/v1/settle", json={"reservation_id": rid, "actual_tokens": 30}, headers=op)
        assert c.post("/authz/v1/snapshot", json=p, headers=op).json() == {"hard_cap": 60, "spent": 30, "reserved": 0}
        assert c.post("/authz/v1/served-usage", json={"model": "m", "prompt_tokens": 3, "completion_tokens": 4},
                      headers=op).json() == {"ok": True}
        code = app.state.ledger.mint_code(40)
        assert c.post("/web/v1/redeem", json={"code": code}, headers=sess).json() == {"added": 40}
        assert c.get("/web/v1/account", headers=sess).json()["allocation_total"] == 140
        ks = c.get("/web/v1/keys", headers=sess).json()["keys"]
        assert c.post(f"/web/v1/keys/{ks[0]['id']}/archive", headers=sess).json() == {"ok": True}
        assert c.get("/web/v1/account").status_code == 401


# ---- bench daemon ---------------------------------------------------------------
from helexa_b200.mesh import benchd  # noqa: E402


def _node_transport(reject_every=3):
    n = {"chat": 0}

    def sse(events):
        return "".join(f"data: {json.dumps(e)}\n\n" for e in events) + "data: [DONE]\n\n"

    def handler(req: httpx.Request):
        p = req.url.path
        if p == "/version":
            return httpx.Response(200, json={"git_sha": "abc123"})
        if p == "/v1/models":
            return httpx.Response(200, json={"data": [{"id": "llm", "capabilities": ["text"]},
                                                      {"id": "img", "capabilities": ["image"]}]})
        if p == "/v1/images/generations":
            return httpx.Response(200, json={"data": [{"b64_json": ""}], "usage": {"helexa_image_units": 2.36}})
        body = json.loads(req.content)
        if body.get("tools"):
            return httpx.Response(200, json={"choices": [{"message": {"tool_calls": [{"id": "c1"}]}}]})
        n["chat"] += 1
        if n["chat"] % reject_every == 0:
            return httpx.Response(429, json={"error": {"code": "rate_limit_exceeded"}})
        evs = [{"choices": [{"delta": {"content": "tok"}}]} for _ in range(5)]
        evs.append({"choices": [], "usage": {"prompt_tokens": 100, "completion_tokens": 5}})
        return httpx.Response(200, text=sse(evs), headers={"content-type": "text/event-stream"})
    return httpx.MockTransport(handler)


def test_bench_daemon_cycle_store_and_api():
    assert 100 * 4 <= len(benchd.build_prompt(100)) <= 100 * 4 + len(benchd.QUESTION)
    store = benchd.Store()
    d = benchd.BenchDaemon([benchd.Target("node", "http://node")], store, transport=_node_transport(reject_every=100))
    asyncio_run = __import__("asyncio").run
    asyncio_run(d.cycle())
    rows = store.runs()
    by = {(r["model"], r["scenario"]): r for r in rows}
    assert set(by) == {("llm", "chat-128"), ("llm", "chat-4096"), ("llm", "concurrency-4"), ("llm", "tool-call"),
                       ("img", "image-512")}
    assert all(r["version"] == "abc123" and r["error"] is None for r in rows)
    assert by[("llm", "chat-128")]["completion_tokens"] == 5 and by[("llm", "chat-128")]["prompt_tokens"] == 100
    assert by[("llm", "concurrency-4")]["concurrency"] == 4 and by[("llm", "concurrency-4")]["completion_tokens"] == 20
    assert by[("llm", "tool-call")]["capability"] == "tool_call"
    assert by[("img", "image-512")]["image_units"] == 2.36
    # admission shedding is counted, not an error
    store2 = benchd.Store()
    d2 = benchd.BenchDaemon([benchd.Target("node", "http://node")], store2, transport=_node_transport(reject_every=2),
                            scenarios=[benchd.Scenario("concurrency-4", "concurrency", 64, 4)])
    asyncio_run(d2.cycle())
    r = store2.runs()[0]
    assert r["rejected"] == 2 and r["error"] is None
    api = benchd.create_bench_api(store)
    with TestClient(api) as c:
        assert c.get("/api/health").json()["runs"] == 5
        s = c.get("/api/summary").json()["summary"]
        assert {x["scenario"] for x in s} >= {"chat-128", "image-512"} and all(x["version"] == "abc123" for x in s)
        assert len(c.get("/api/series", params={"model": "llm", "scenario": "chat-128"}).json()["points"]) == 1
        assert len(c.get("/api/runs", params={"limit": 2}).json()["runs"]) == 2


# ---- ACP bridge -----------------------------------------------------------------
from helexa_b200.mesh import acp  # noqa: E402


class _ScriptProvider:
    def __init__(self, rounds):
        self.rounds, self.seen = list(rounds), []

    async def stream(self, messages, tools):
        self.seen.append([dict(m) for m in messages])
        text, calls = self.rounds.pop(0)
        for piece in text:
            yield "text", piece
        yield "tool_calls", calls


def _drive(provider, script, allow=True):
    """Run the agent against an in-memory editor; `script` is the list of requests the
    editor sends. Returns every message the agent wrote and the editor's files."""
    import asyncio
    files = {"/w/a.py": "x = 1\n"}
    out = []

    async def main():
        reader = asyncio.StreamReader()
        agent = None

        def write(b):
            msg = json.loads(b)
            out.append(msg)
            if "method" in msg and "id" in msg:  # a request to the editor
                m, p = msg["method"], msg["params"]
                if m == "fs/read_text_file":
                    res = {"content": files[p["path"]]}
                elif m == "fs/write_text_file":
                    files[p["path"]] = p["content"]
                    res = None
                elif m == "session/request_permission":
                    res = {"outcome": {"outcome": "selected", "optionId": "allow" if allow else "reject"}}
                else:
                    res = {}
                reader.feed_data((json.dumps({"jsonrpc": "2.0", "id": msg["id"], "result": res}) + "\n").encode())

        agent = acp.AcpAgent(provider, reader, write)
        task = asyncio.create_task(agent.serve())
        for req in script:
            if callable(req):
                req = req(out)
            reader.feed_data((json.dumps(req) + "\n").encode())
            for _ in range(50):
                await asyncio.sleep(0.005)
        reader.feed_eof()
        await task

    asyncio.run(main())
    return out, files


def _sid(out):
    return next(m["result"]["sessionId"] for m in out if m.get("id") == 2 and "result" in m)


def test_acp_prompt_tool_loop_and_permissions():
    rounds = [("Looking", [{"id": "c1", "name": "read_file", "arguments": json.dumps({"path": "/w/a.py"})}]),
              ("", [{"id": "c2", "name": "edit_file",
                     "arguments": json.dumps({"path": "/w/a.py", "old_text": "x = 1", "new_text": "x = 2"})}]),
              ("Done.", [])]
    prov = _ScriptProvider(rounds)
    out, files = _drive(prov, [
        {"jsonrpc": "2.0", "id": 1, "method": "initialize", "params": {"protocolVersion": 1}},
        {"jsonrpc": "2.0", "id": 2, "method": "session/new", "params": {"cwd": "/w"}},
        lambda o: {"jsonrpc": "2.0", "id": 3, "method": "session/prompt",
                   "params": {"sessionId": _sid(o), "prompt": [{"type": "text", "text": "bump x"}]}},
        {"jsonrpc": "2.0", "id": 4, "method": "nope/nope", "params": {}},
    ])
    res = {m["id"]: m for m in out if "id" in m and ("result" in m or "error" in m)}
    assert res[1]["result"]["protocolVersion"] == 1
    assert res[3]["result"] == {"stopReason": "end_turn"}
    assert res[4]["error"]["code"] == -32601
    assert files["/w/a.py"] == "x = 2\n"
    ups = [m["params"]["update"] for m in out if m.get("method") == "session/update"]
    assert [u["sessionUpdate"] for u in ups if u["sessionUpdate"] != "agent_message_chunk"] == \
        ["tool_call", "tool_call_update", "tool_call", "tool_call_update"]
    assert all(u["status"] == "completed" for u in ups if u["sessionUpdate"] == "tool_call_update")
    text = "".join(u["content"]["text"] for u in ups if u["sessionUpdate"] == "agent_message_chunk")
    assert text == "LookingDone."
    assert any(m.get("method") == "session/request_permission" for m in out)  # edit is gated in default mode
    # the tool result went back to the model
    assert prov.seen[1][-1] == {"role": "tool", "tool_call_id": "c1", "content": "x = 1\n"}


def test_acp_rejected_permission_and_bypass_mode():
    rounds = [("", [{"id": "c1", "name": "write_file", "arguments": json.dumps({"path": "/w/a.py", "content": "y"})}]),
              ("ok", [])]
    out, files = _drive(_ScriptProvider(rounds), [
        {"jsonrpc": "2.0", "id": 1, "method": "initialize", "params": {}},
        {"jsonrpc": "2.0", "id": 2, "method": "session/new", "params": {"cwd": "/w"}},
        lambda o: {"jsonrpc": "2.0", "id": 3, "method": "session/prompt",
                   "params": {"sessionId": _sid(o), "prompt": [{"type": "text", "text": "w"}]}},
    ], allow=False)
    assert files["/w/a.py"] == "x = 1\n"
    ups = [m["params"]["update"] for m in out if m.get("method") == "session/update"]
    assert [u["status"] for u in ups if u["sessionUpdate"] == "tool_call_update"] == ["failed"]
    rounds = [("", [{"id": "c1", "name": "write_file", "arguments": json.dumps({"path": "/w/a.py", "content": "y"})}]),
              ("ok", [])]
    out, files = _drive(_ScriptProvider(rounds), [
        {"jsonrpc": "2.0", "id": 1, "method": "initialize", "params": {}},
        {"jsonrpc": "2.0", "id": 2, "method": "session/new", "params": {"cwd": "/w"}},
        lambda o: {"jsonrpc": "2.0", "id": 5, "method": "session/set_mode",
                   "params": {"sessionId": _sid(o), "modeId": "bypassPermissions"}},
        lambda o: {"jsonrpc": "2.0", "id": 3, "method": "session/prompt",
                   "params": {"sessionId": _sid(o), "prompt": [{"type": "text", "text": "w"}]}},
    ])
    assert files["/w/a.py"] == "y"
    assert not any(m.get("method") == "session/request_permission" for m in out)


def test_acp_openai_provider_parses_streamed_tool_calls():
    import asyncio
    evs = [{"choices": [{"delta": {"content": "Hi"}}]},
           {"choices": [{"delta": {"tool_calls": [{"index": 0, "id": "t1", "function": {"name": "read_",
                                                                                         "arguments": "{\"pa"}}]}}]},
           {"choices": [{"delta": {"tool_calls": [{"index": 0, "function": {"name": "file",
                                                                             "arguments": "th\": \"/x\"}"}}]}}]}]
    body = "".join(f"data: {json.dumps(e)}\n\n" for e in evs) + "data: [DONE]\n\n"
    tr = httpx.MockTransport(lambda r: httpx.Response(200, text=body, headers={"content-type": "text/event-stream"}))
    p = acp.OpenAIProvider("http://gw/v1", "m", transport=tr)

    async def run():
        return [x async for x in p.stream([], acp.TOOLS)]

    got = asyncio.run(run())
    assert got == [("text", "Hi"), ("tool_calls", [{"id": "t1", "name": "read_file", "arguments": "{\"path\": \"/x\"}"}])]


def test_cli_lists_mesh_services():
    import subprocess
    import sys
    out = subprocess.run([sys.executable, "-m", "helexa_b200.cli", "--help"], capture_output=True, text=True,
                         timeout=120).stdout
    for cmd in ("node", "serve", "status", "router", "tools", "upstream", "bench", "acp", "portal"):
        assert cmd in out


# ---- document portal ---------------------------------------------------------------
from helexa_b200.mesh import portal as pt  # noqa: E402


def test_portal_invites_grants_audit_watermark():
    L = up.Ledger()
    P = pt.Portal(L)
    P.create_round("seed", "Seed round")
    v1 = P.put_document("seed", "deck", "Deck", "Para one.\n\n<script>x</script>")
    auto = P.mint_invite("seed", "partners", auto_grant=True)
    manual = P.mint_invite("seed", "public")
    dead = P.mint_invite("seed", "old")
    P.revoke_invite(dead)
    app = pt.create_portal(P)
    with TestClient(app) as c:
        assert "Sign in" in c.get("/").text
        assert "Sign in" in c.get("/r/seed/deck").text  # no session: only the sign-in form
        # an invite before sign-in is remembered and applied at registration
        r = c.get(f"/i/{auto}", follow_redirects=False)
        assert r.status_code == 303 and r.headers["location"] == "/register"
        r = c.post("/register", data={"email": "ann@fund.io", "password": "long enough pw"})
        assert "Seed round" in r.text
        page = c.get("/r/seed/deck").text
        assert "ann@fund.io" in page and "&lt;script&gt;" in page and "<script>x" not in page
        assert f"version {v1}" in page
        c.get("/signout")
        assert "Sign in" in c.get("/").text
    with TestClient(app) as c2:  # a forwarded, non-auto code yields a pending, named grant
        c2.post("/register", data={"email": "bob@x.io", "password": "another password"})
        c2.get(f"/i/{manual}")
        assert "awaiting approval" in c2.get("/").text
        assert "not available" in c2.get("/r/seed/deck").text
        bob = L.check_password("bob@x.io", "another password")
        P.set_grant(bob, "seed", "active")
        assert "Para one." in c2.get("/r/seed/deck").text
        c2.get(f"/i/{dead}")  # a revoked code changes nothing
        P.set_grant(bob, "seed", "revoked")
        assert "not available" in c2.get("/r/seed/deck").text
    assert c2.post("/signin", data={"email": "bob@x.io", "password": "wrong"}).status_code == 200
    log = P.audit_log()
    views = [(e["email"], e["document"], e["version"]) for e in log if e["kind"] == "view"]
    assert views == [("ann@fund.io", "deck", v1), ("bob@x.io", "deck", v1)]
    assert any(e["kind"] == "denied" and e["email"] == "bob@x.io" for e in log)
    # a portal session is not a ledger session and vice versa
    assert L.session_account("nope") is None and P.session_account(L.new_session(bob)) is None
