"""Gateway HTTP app: OpenAI / Anthropic surface in front of a fleet of nodes.

Routes (cortex-gateway/src/handlers.rs:21-31): /v1/chat/completions /v1/completions
/v1/responses /v1/messages /v1/images/generations /v1/models /health / and a
Prometheus /metrics. Bearer keys resolve to principals; the gateway strips any
client-supplied `x-helexa-*` headers and stamps its own (auth.rs anti-spoofing).
Requests are proxied verbatim (SSE forwarded as it arrives), with the model rewritten
when an alias was used; metrics count requests, latency, TTFT and tokens
(metrics.rs:99-140).
"""
from __future__ import annotations

import asyncio
import json
import time

import httpx
from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, Response, StreamingResponse
from prometheus_client import CollectorRegistry, Counter, Histogram, generate_latest

from ..server.wire import error_body
from .budget import BudgetExceeded, BudgetLedger, Cap, SSEUsage, estimate_prompt_tokens, reservation_estimate
from .core import Catalogue, NodeState, NoRoute, Router


class Metrics:
    def __init__(self):
        self.reg = CollectorRegistry()
        self.requests = Counter("cortex_requests_total", "requests", ["model", "status"], registry=self.reg)
        self.duration = Histogram("cortex_request_duration_seconds", "request latency", ["model"], registry=self.reg)
        self.ttft = Histogram("cortex_time_to_first_token_seconds", "time to first token", ["model"],
                              registry=self.reg)
        self.tokens = Counter("cortex_completion_tokens_total", "completion tokens", ["model"], registry=self.reg)
        self.cold = Counter("cortex_cold_starts_total", "cold loads", ["model"], registry=self.reg)
        self.evictions = Counter("cortex_evictions_total", "evictions", ["model"], registry=self.reg)
        self.principal_requests = Counter("cortex_principal_requests_total", "requests per principal",
                                          ["principal", "model"], registry=self.reg)
        self.principal_tokens = Counter("cortex_principal_tokens_total", "tokens per principal",
                                        ["principal", "model", "kind"], registry=self.reg)


def create_gateway(catalogue: Catalogue, nodes: list[NodeState], api_keys: dict[str, str] | None = None,
                   require_auth: bool = False, poll_interval_s: float = 10.0, transport=None,
                   entitlements: dict[str, set[str]] | None = None,
                   budgets: dict[str, Cap] | None = None) -> FastAPI:
    """`entitlements`: principal -> models it may use (a principal absent from the map,
    and anonymous callers, may use every model). Usage is metered per principal
    (anonymous callers as "anonymous") into `/metrics` and `GET /usage`. `budgets`:
    principal -> token cap, enforced by reserve -> settle (`gateway/budget.py`)."""
    app = FastAPI(title="helexa-b200 gateway")
    router = Router(catalogue, nodes)
    metrics = Metrics()
    client = httpx.AsyncClient(timeout=httpx.Timeout(600.0, connect=10.0), transport=transport)
    app.state.router = router
    app.state.metrics = metrics
    app.state.client = client
    usage: dict[str, dict[str, int]] = {}
    app.state.usage = usage
    ledger = BudgetLedger(budgets)
    app.state.ledger = ledger

    def _meter(principal: str | None, model: str, prompt: int = 0, completion: int = 0, request: bool = False):
        who = principal or "anonymous"
        u = usage.setdefault(who, {"requests": 0, "prompt_tokens": 0, "completion_tokens": 0})
        if request:
            u["requests"] += 1
            metrics.principal_requests.labels(who, model).inc()
        u["prompt_tokens"] += prompt
        u["completion_tokens"] += completion
        if prompt:
            metrics.principal_tokens.labels(who, model, "prompt").inc(prompt)
        if completion:
            metrics.principal_tokens.labels(who, model, "completion").inc(completion)

    async def poll_once():
        for n in list(router.nodes.values()):
            try:
                ms = (await client.get(n.url + "/models")).json().get("models", [])
                hl = (await client.get(n.url + "/health")).json()
                disc = (await client.get(n.url + "/discovery")).json()
                free = sum(d.get("memory_free_mb", 0) for d in disc.get("devices", []))
                router.observe(n.name, ms, hl, free)
            except Exception:
                router.observe(n.name, None, None)

    app.state.poll_once = poll_once

    @app.on_event("startup")
    async def _start():
        async def loop():
            while True:
                await poll_once()
                await asyncio.sleep(poll_interval_s)
        app.state.poller = asyncio.get_running_loop().create_task(loop())

    @app.on_event("shutdown")
    async def _stop():
        app.state.poller.cancel()
        await client.aclose()

    def _principal(request: Request) -> tuple[str | None, JSONResponse | None]:
        auth = request.headers.get("authorization", "")
        key = auth[7:] if auth.lower().startswith("bearer ") else None
        if key and api_keys and key in api_keys:
            return api_keys[key], None
        if require_auth:
            return None, JSONResponse(error_body("invalid or missing API key", "invalid_api_key"), 401)
        return None, None

    async def _proxy(request: Request, path: str):
        body = await request.json()
        principal, err = _principal(request)
        if err is not None:
            return err
        requested = body.get("model", "")
        if principal and entitlements and principal in entitlements:
            target = catalogue.resolve(requested)
            if requested not in entitlements[principal] and target not in entitlements[principal]:
                return JSONResponse(error_body(f"principal is not entitled to model {requested!r}",
                                               "model_not_entitled"), 403)
        t0 = time.monotonic()
        try:
            dec = router.route(requested)
        except NoRoute as e:
            metrics.requests.labels(requested, str(e.status)).inc()
            h = {"Retry-After": str(e.retry_after)} if e.retry_after else None
            return JSONResponse(error_body(str(e), e.code), e.status, headers=h)
        # fail-fast prompt pre-validation against the advertised context (the node stays
        # the exact limit; the estimate under-counts, so only gross overages stop here)
        lim = (dec.node.models.get(dec.model_id) or {}).get("limit") or {}
        est = estimate_prompt_tokens(body)
        if isinstance(lim.get("context"), int) and est > lim["context"]:
            metrics.requests.labels(dec.model_id, "400").inc()
            return JSONResponse(error_body(f"prompt is about {est} tokens; {dec.model_id} accepts at most "
                                           f"{lim['context']}", "context_length_exceeded"), 400)
        try:
            resv = ledger.reserve(principal, reservation_estimate(body, lim.get("output")))
        except BudgetExceeded as e:
            metrics.requests.labels(dec.model_id, "429").inc()
            h = {"Retry-After": str(e.retry_after)} if e.retry_after else None
            return JSONResponse(error_body(str(e), e.code), 429, headers=h)
        handoff = {"stream": False}
        try:
            return await _dispatch(request, path, body, principal, requested, dec, t0, resv, handoff)
        finally:
            if not handoff["stream"]:  # a streamed response settles when its relay ends
                ledger.release(resv)  # no-op once settled

    async def _dispatch(request, path, body, principal, requested, dec, t0, resv, handoff):
        if dec.action == "cold_load":
            for victim in dec.evict:
                await client.post(dec.node.url + "/models/unload", json={"model_id": victim})
                dec.node.models.pop(victim, None)
                metrics.evictions.labels(victim).inc()
            entry = catalogue.entries[dec.model_id]
            spec = dict(entry.load_spec, model_id=dec.model_id, source=entry.source,
                        tensor_parallel=entry.tensor_parallel)
            r = await client.post(dec.node.url + "/models/load", json=spec)
            metrics.cold.labels(dec.model_id).inc()
            if r.status_code != 200:
                return JSONResponse(r.json(), r.status_code)
            dec.node.models[dec.model_id] = {"id": dec.model_id, "status": "loaded"}
        body["model"] = dec.model_id
        _meter(principal, dec.model_id, request=True)
        headers = {k: v for k, v in request.headers.items()
                   if not k.lower().startswith("x-helexa-") and k.lower() not in ("host", "content-length",
                                                                                   "authorization")}
        if principal:
            headers["x-helexa-account"] = principal
        url = dec.node.url + path
        if body.get("stream"):
            req = client.build_request("POST", url, json=body, headers=headers)
            resp = await client.send(req, stream=True)

            async def relay():
                first = True
                seen = SSEUsage()
                try:
                    async for chunk in resp.aiter_bytes():
                        if first:
                            metrics.ttft.labels(dec.model_id).observe(time.monotonic() - t0)
                            first = False
                        seen.feed(chunk)
                        yield chunk
                finally:
                    await resp.aclose()
                    metrics.requests.labels(dec.model_id, str(resp.status_code)).inc()
                    metrics.duration.labels(dec.model_id).observe(time.monotonic() - t0)
                    metrics.tokens.labels(dec.model_id).inc(seen.completion)
                    _meter(principal, dec.model_id, prompt=seen.prompt, completion=seen.completion)
                    if seen.seen:
                        ledger.settle(resv, seen.prompt + seen.completion)
                    else:
                        ledger.release(resv)
            handoff["stream"] = True
            return StreamingResponse(relay(), status_code=resp.status_code,
                                     media_type=resp.headers.get("content-type", "text/event-stream"))
        r = await client.post(url, json=body, headers=headers)
        metrics.requests.labels(dec.model_id, str(r.status_code)).inc()
        metrics.duration.labels(dec.model_id).observe(time.monotonic() - t0)
        try:
            j = r.json()
            rep = j.get("usage") or {}
            metrics.tokens.labels(dec.model_id).inc(rep.get("completion_tokens", rep.get("output_tokens", 0)))
            pt = int(rep.get("prompt_tokens", rep.get("input_tokens", 0)) or 0)
            ct = int(rep.get("completion_tokens", rep.get("output_tokens", 0)) or 0)
            _meter(principal, dec.model_id, prompt=pt, completion=ct)
            if rep:
                ledger.settle(resv, pt + ct)
            if requested != dec.model_id and isinstance(j, dict) and "model" in j:
                j["model"] = requested
            return JSONResponse(j, r.status_code, headers={k: v for k, v in r.headers.items()
                                                           if k.lower() == "retry-after"})
        except json.JSONDecodeError:
            return Response(r.content, r.status_code)

    for path in ("/v1/chat/completions", "/v1/completions", "/v1/responses", "/v1/messages",
                 "/v1/images/generations"):
        async def handler(request: Request, _p=path):
            return await _proxy(request, _p)
        app.post(path)(handler)

    @app.get("/v1/models")
    async def models():
        data = []
        for mid, e in catalogue.entries.items():
            loaded = [n.name for n in router.nodes.values() if n.models.get(mid, {}).get("status") == "loaded"]
            lim = next((n.models[mid].get("limit") for n in router.nodes.values() if mid in n.models), None)
            caps = sorted({c for n in router.nodes.values() if n.models.get(mid, {}).get("status") == "loaded"
                           for c in n.models[mid].get("capabilities", [])})
            item = {"id": mid, "object": "model", "owned_by": "helexa", "aliases": e.aliases,
                    "loaded_on": loaded, "limit": lim, "loaded": bool(loaded),
                    # a catalogue entry can be cold-loaded on any healthy node
                    "feasible_on": [n.name for n in router.nodes.values() if n.healthy],
                    "capabilities": caps}
            if e.cost_input_per_mtok is not None or e.cost_output_per_mtok is not None:
                item["cost"] = {"input_per_mtok": e.cost_input_per_mtok, "output_per_mtok": e.cost_output_per_mtok}
            data.append(item)
        return {"object": "list", "data": data}

    @app.get("/usage")
    async def usage_report():
        out = {}
        for who, u in usage.items():
            b = ledger.snapshot(who)
            out[who] = dict(u, budget=b) if b else u
        return {"principals": out}

    @app.get("/health")
    async def health():
        ns = list(router.nodes.values())
        return {"status": "ok", "nodes": {"healthy": sum(1 for n in ns if n.healthy), "total": len(ns),
                                          "by_name": {n.name: {"healthy": n.healthy, "models": list(n.models)}
                                                      for n in ns}}}

    @app.get("/")
    async def root():
        return {"service": "helexa-b200 gateway"}

    @app.get("/ui")
    async def ui():
        """Browser chat client (static page; it calls this gateway's own API)."""
        import os
        from fastapi.responses import HTMLResponse
        with open(os.path.join(os.path.dirname(__file__), "static", "chat.html"), encoding="utf-8") as f:
            return HTMLResponse(f.read())

    @app.get("/metrics")
    async def prom():
        return Response(generate_latest(metrics.reg), media_type="text/plain; version=0.0.4")

    return app
