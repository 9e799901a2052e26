"""Federation ingress: one OpenAI / Anthropic endpoint in front of several operators'
gateways ("cortexes"), as the reference's helexa-router does (crates/helexa-router:
poller.rs, dispatch.rs, catalogue.rs, handlers.rs).

* Poller: every `poll_interval_s` each cortex's `/v1/models` (entries with `loaded`,
  `feasible_on`, `limit`, `cost`, `capabilities`) and `/health` (`nodes.healthy`) are
  read; a cortex is unreachable after 3 consecutive failed polls (one failure keeps the
  last topology, so a blip does not drop capacity).
* Selection for a model: cortexes whose entry is loaded or feasible, reachable, ranked
  by (loaded first, same region first, more healthy nodes first, name). Unknown
  everywhere -> 404 `model_not_found`; known but nowhere reachable -> 503 with
  Retry-After.
* Dispatch forwards the body verbatim (the model rewritten when a tier alias was used)
  and streams the answer back; a cortex that cannot be reached is failed over to the
  next candidate.
* `/v1/models` merges every reachable cortex's entries: loaded if loaded anywhere,
  `feasible_on` = the cortexes, capabilities unioned, the tightest context limit and
  the cheapest cost.
"""
from __future__ import annotations

import asyncio
import json
import time
from dataclasses import dataclass, field

import httpx
from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, StreamingResponse

from ..server.wire import error_body

POLL_FAILURE_THRESHOLD = 3
RETRY_AFTER_S = 5


@dataclass
class CortexEndpoint:
    name: str
    endpoint: str
    region: str | None = None


@dataclass
class CortexTopology:
    models: dict = field(default_factory=dict)   # model id -> entry dict
    reachable: bool = False
    consecutive_failures: int = 0
    healthy_nodes: int = 0
    last_poll: float | None = None


@dataclass
class RouterConfig:
    cortexes: list[CortexEndpoint]
    aliases: dict[str, str] = field(default_factory=dict)
    region: str | None = None
    poll_interval_s: float = 10.0

    @classmethod
    def from_dict(cls, d: dict) -> "RouterConfig":
        r = d.get("router", {})
        return cls(cortexes=[CortexEndpoint(**c) for c in d.get("cortexes", [])], aliases=d.get("aliases", {}),
                   region=r.get("region"), poll_interval_s=float(r.get("poll_interval_secs", 10)))

    @classmethod
    def load(cls, path: str) -> "RouterConfig":
        import tomllib
        with open(path, "rb") as f:
            return cls.from_dict(tomllib.load(f))


def entry_feasible(e: dict) -> bool:
    return bool(e.get("loaded")) or bool(e.get("feasible_on"))


class RouterState:
    def __init__(self, cfg: RouterConfig):
        self.cfg = cfg
        self.topology = {c.name: CortexTopology() for c in cfg.cortexes}
        self.by_name = {c.name: c for c in cfg.cortexes}

    # ---- poller ----
    def observe(self, name: str, models: list | None, healthy_nodes: int | None = None):
        t = self.topology.get(name)
        if t is None:
            return
        if models is None:
            t.consecutive_failures += 1
            if t.consecutive_failures >= POLL_FAILURE_THRESHOLD:
                t.reachable = False
            return
        t.models = {m["id"]: m for m in models if "id" in m}
        t.reachable = True
        t.consecutive_failures = 0
        t.last_poll = time.time()
        if healthy_nodes is not None:
            t.healthy_nodes = healthy_nodes

    async def poll_once(self, client: httpx.AsyncClient):
        async def one(c: CortexEndpoint):
            try:
                r = await client.get(c.endpoint + "/v1/models", timeout=5.0)
                r.raise_for_status()
                models = r.json().get("data", [])
            except Exception:
                self.observe(c.name, None)
                return
            healthy = None
            try:
                h = (await client.get(c.endpoint + "/health", timeout=5.0)).json()
                healthy = int(h.get("nodes", {}).get("healthy", 0))
            except Exception:
                pass
            self.observe(c.name, models, healthy)

        await asyncio.gather(*(one(c) for c in self.cfg.cortexes))

    # ---- selection ----
    def select(self, model: str):
        """('candidates', [CortexEndpoint]) | ('unknown', None) | ('unreachable', None)"""
        ranked, known = [], False
        for name, t in self.topology.items():
            e = t.models.get(model)
            if e is None or not entry_feasible(e):
                continue
            known = True
            if not t.reachable or name not in self.by_name:
                continue
            ep = self.by_name[name]
            region_match = self.cfg.region is not None and ep.region == self.cfg.region
            ranked.append(((not e.get("loaded"), not region_match, -t.healthy_nodes, name), ep))
        if not ranked:
            return ("unreachable", None) if known else ("unknown", None)
        ranked.sort(key=lambda x: x[0])
        return "candidates", [ep for _, ep in ranked]

    # ---- catalogue ----
    def aggregate_models(self) -> list[dict]:
        merged: dict[str, dict] = {}
        for name in sorted(self.topology):
            t = self.topology[name]
            if not t.reachable:
                continue
            for e in t.models.values():
                if not entry_feasible(e):
                    continue
                loc = [{"node": name, "status": "loaded"}] if e.get("loaded") else []
                acc = merged.get(e["id"])
                if acc is None:
                    merged[e["id"]] = {"id": e["id"], "object": "model", "created": e.get("created", 0),
                                       "owned_by": e.get("owned_by", "helexa"), "loaded": bool(e.get("loaded")),
                                       "feasible_on": [name], "locations": loc,
                                       "capabilities": list(e.get("capabilities", [])), "limit": e.get("limit"),
                                       "cost": e.get("cost")}
                    continue
                acc["loaded"] |= bool(e.get("loaded"))
                acc["feasible_on"].append(name)
                acc["locations"] += loc
                for c in e.get("capabilities", []):
                    if c not in acc["capabilities"]:
                        acc["capabilities"].append(c)
                lim = e.get("limit")
                if lim and (not acc["limit"] or lim.get("context", 1 << 62) < acc["limit"].get("context", 1 << 62)):
                    acc["limit"] = lim
                cost = e.get("cost")
                if cost and (not acc["cost"] or _price(cost) < _price(acc["cost"])):
                    acc["cost"] = cost
        return [merged[k] for k in sorted(merged)]


def _price(c: dict) -> float:
    return float(c.get("input_per_mtok") or 0) + float(c.get("output_per_mtok") or 0)


def create_router(cfg: RouterConfig, transport=None, poll: bool = True) -> FastAPI:
    app = FastAPI(title="helexa-b200 federation router")
    state = RouterState(cfg)
    client = httpx.AsyncClient(timeout=httpx.Timeout(600.0, connect=10.0), transport=transport)
    app.state.router = state
    app.state.client = client

    async def poll_once():
        await state.poll_once(client)

    app.state.poll_once = poll_once

    @app.on_event("startup")
    async def _start():
        if not poll:
            return

        async def loop():
            while True:
                await poll_once()
                await asyncio.sleep(cfg.poll_interval_s)

        app.state.poller = asyncio.create_task(loop())

    @app.on_event("shutdown")
    async def _stop():
        t = getattr(app.state, "poller", None)
        if t:
            t.cancel()
        await client.aclose()

    async def dispatch(path: str, request: Request):
        raw = await request.body()
        try:
            body = json.loads(raw)
            model = body.get("model")
        except (ValueError, AttributeError):
            body, model = None, None
        if not isinstance(model, str):
            return JSONResponse(error_body("missing 'model' field in request body", "missing_model_field"), 400)
        real = cfg.aliases.get(model)
        if real is not None:
            body["model"] = real
            model, raw = real, json.dumps(body).encode()
        kind, cands = state.select(model)
        if kind == "unknown":
            return JSONResponse(error_body(f"no operator serves model '{model}'", "model_not_found"), 404)
        if kind == "unreachable":
            return JSONResponse(error_body(f"model '{model}' is temporarily unavailable on all operators",
                                           "service_unavailable"), 503, headers={"Retry-After": str(RETRY_AFTER_S)})
        fwd = {k: v for k, v in request.headers.items() if k.lower() in ("authorization", "content-type", "accept",
                                                                         "x-include-thinking", "anthropic-version")}
        for ep in cands:
            try:
                req = client.build_request("POST", ep.endpoint + path, content=raw, headers=fwd)
                resp = await client.send(req, stream=True)
            except httpx.TransportError:
                continue  # fail over to the next operator

            async def relay(resp=resp):
                try:
                    async for chunk in resp.aiter_bytes():
                        yield chunk
                finally:
                    await resp.aclose()

            headers = {k: v for k, v in resp.headers.items()
                       if k.lower() in ("content-type", "retry-after", "cache-control")}
            return StreamingResponse(relay(), status_code=resp.status_code, headers=headers)
        return JSONResponse(error_body(f"all operators able to serve '{model}' are unreachable",
                                       "service_unavailable"), 503, headers={"Retry-After": str(RETRY_AFTER_S)})

    for path in ("/v1/chat/completions", "/v1/completions", "/v1/responses", "/v1/messages",
                 "/v1/images/generations"):
        async def handler(request: Request, _p=path):
            return await dispatch(_p, request)
        app.add_api_route(path, handler, methods=["POST"])

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": state.aggregate_models()}

    @app.get("/health")
    @app.get("/")
    async def health():
        return {"status": "ok", "cortexes": {"configured": len(cfg.cortexes),
                                             "reachable": sum(1 for t in state.topology.values() if t.reachable)}}

    return app


def main(argv=None):
    import argparse

    import uvicorn
    ap = argparse.ArgumentParser(description="helexa-b200 federation router")
    ap.add_argument("--config", required=True, help="TOML: [router] listen/region/poll_interval_secs, "
                                                     "[[cortexes]] name/endpoint/region, [aliases]")
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=8088)
    a = ap.parse_args(argv)
    uvicorn.run(create_router(RouterConfig.load(a.config)), host=a.host, port=a.port)


if __name__ == "__main__":
    main()
