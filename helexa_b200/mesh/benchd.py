"""Continuous, version-aware benchmark daemon: on an interval it reads each target's
build (`/version`) and served models (`/v1/models`), runs the scenarios that apply to
each model through the public streaming API, and stores every run in SQLite keyed by
target, build and model, so a regression shows up as a step in a series (the
reference's crates/helexa-bench: scenario.rs, store.rs, report.rs, api.rs).

Scenarios:
* chat latency at a prompt size: TTFT (request -> first content chunk), decode tok/s
  (usage completion tokens over the first -> last chunk window, or chunk rate when the
  server reports no usage), total time;
* concurrency: N identical streams at once: aggregate tok/s over the burst, p95 TTFT,
  streams shed by admission control (429 / 503);
* capability probe: does a tool-call request come back as a tool call;
* image latency (image models only): one generation, wall time and image units.

HTTP (`create_bench_api`): /api/health, /api/summary (median per build, model and
scenario), /api/series?model=&scenario= (time-ordered), /api/runs?limit=.
"""
from __future__ import annotations

import asyncio
import json
import sqlite3
import statistics
import threading
import time
from dataclasses import dataclass, field

import httpx
from fastapi import FastAPI

FILLER = ("The quick brown fox jumps over the lazy dog while the committee reviews the quarterly "
          "figures and the weather turns from clear to overcast over the harbour. ")
QUESTION = "\n\nIn one short paragraph, summarise the text above."


def build_prompt(approx_tokens: int) -> str:
    """About `approx_tokens` tokens of filler (4 characters per token) and a question."""
    n = max(16, approx_tokens) * 4
    return (FILLER * (n // len(FILLER) + 1))[:n] + QUESTION


@dataclass
class Metrics:
    ttft_s: float = 0.0
    decode_tps: float | None = None
    total_s: float = 0.0
    prompt_tokens: int | None = None
    completion_tokens: int = 0
    concurrency: int | None = None
    ttft_p95_s: float | None = None
    rejected: int | None = None
    capability: str | None = None
    image_units: float | None = None


class AdmissionRejected(Exception):
    pass


async def stream_and_measure(client: httpx.AsyncClient, url: str, payload: dict) -> Metrics:
    t0 = time.monotonic()
    first = last = None
    chunks, usage = 0, None
    async with client.stream("POST", url, json=payload) as r:
        if r.status_code in (429, 503):
            raise AdmissionRejected(f"status {r.status_code}")
        if r.status_code != 200:
            raise RuntimeError(f"status {r.status_code}: {(await r.aread())[:200]!r}")
        async for line in r.aiter_lines():
            if not line.startswith("data: ") or line[6:].strip() == "[DONE]":
                continue
            try:
                ev = json.loads(line[6:])
            except ValueError:
                continue  # keep-alive or non-JSON frame
            if ev.get("usage"):
                usage = ev["usage"]
            for ch in ev.get("choices", []):
                d = ch.get("delta", {})
                if d.get("content") or d.get("reasoning_content") or d.get("tool_calls"):
                    now = time.monotonic()
                    first = first or now
                    last = now
                    chunks += 1
    end = time.monotonic()
    m = Metrics(total_s=end - t0, ttft_s=(first or end) - t0)
    if usage:
        m.prompt_tokens = usage.get("prompt_tokens")
        m.completion_tokens = int(usage.get("completion_tokens", 0))
    else:
        m.completion_tokens = chunks
    window = (last - first) if first and last else 0.0
    if window > 0.2 and m.completion_tokens > 1:
        m.decode_tps = (m.completion_tokens - 1) / window
    elif window > 0.2:
        m.decode_tps = chunks / window
    return m


@dataclass
class Scenario:
    id: str
    kind: str                     # chat | concurrency | capability | image
    prompt_tokens: int = 128
    concurrency: int = 1

    def applies_to(self, caps: list[str]) -> bool:
        return (self.kind == "image") == ("image" in caps)


DEFAULT_SCENARIOS = [Scenario("chat-128", "chat", 128), Scenario("chat-4096", "chat", 4096),
                     Scenario("concurrency-4", "concurrency", 512, 4), Scenario("tool-call", "capability", 64),
                     Scenario("image-512", "image")]


async def run_scenario(client: httpx.AsyncClient, base: str, model: str, sc: Scenario, max_tokens: int = 128,
                       timeout_s: float = 300.0) -> Metrics:
    chat_url = base + "/v1/chat/completions"
    payload = {"model": model, "stream": True, "max_tokens": max_tokens, "temperature": 0,
               "stream_options": {"include_usage": True},
               "messages": [{"role": "user", "content": build_prompt(sc.prompt_tokens)}]}
    if sc.kind == "chat":
        return await asyncio.wait_for(stream_and_measure(client, chat_url, payload), timeout_s)
    if sc.kind == "concurrency":
        t0 = time.monotonic()
        res = await asyncio.gather(*(asyncio.wait_for(stream_and_measure(client, chat_url, payload), timeout_s)
                                     for _ in range(sc.concurrency)), return_exceptions=True)
        window = time.monotonic() - t0
        ok = [r for r in res if isinstance(r, Metrics)]
        rejected = sum(1 for r in res if isinstance(r, AdmissionRejected))
        if not ok:
            raise RuntimeError(f"all {sc.concurrency} concurrent streams failed ({rejected} shed by admission)")
        ttfts = sorted(m.ttft_s for m in ok)
        tot = sum(m.completion_tokens for m in ok)
        return Metrics(ttft_s=statistics.median(ttfts), ttft_p95_s=ttfts[min(len(ttfts) - 1, int(0.95 * len(ttfts)))],
                       decode_tps=tot / window if window > 0 else None, total_s=window, completion_tokens=tot,
                       concurrency=sc.concurrency, rejected=rejected)
    if sc.kind == "capability":
        tool = {"type": "function", "function": {"name": "get_weather", "description": "weather for a city",
                                                 "parameters": {"type": "object",
                                                                "properties": {"city": {"type": "string"}}}}}
        body = {"model": model, "max_tokens": max_tokens, "temperature": 0, "tools": [tool],
                "messages": [{"role": "user", "content": "What is the weather in Paris? Use the tool."}]}
        t0 = time.monotonic()
        r = await client.post(chat_url, json=body, timeout=timeout_s)
        msg = (r.json().get("choices") or [{}])[0].get("message", {})
        return Metrics(total_s=time.monotonic() - t0, capability="tool_call" if msg.get("tool_calls") else "text")
    if sc.kind == "image":
        t0 = time.monotonic()
        r = await client.post(base + "/v1/images/generations", timeout=timeout_s,
                              json={"model": model, "prompt": "a lighthouse at dusk", "size": "512x512", "seed": 1})
        if r.status_code != 200:
            raise RuntimeError(f"status {r.status_code}")
        return Metrics(total_s=time.monotonic() - t0, image_units=r.json().get("usage", {}).get("helexa_image_units"))
    raise ValueError(sc.kind)


class Store:
    COLUMNS = [("ts", "REAL"), ("target", "TEXT"), ("endpoint", "TEXT"), ("version", "TEXT"), ("model", "TEXT"),
               ("scenario", "TEXT"), ("prompt_size", "INTEGER"), ("ttft_s", "REAL"), ("decode_tps", "REAL"),
               ("total_s", "REAL"), ("prompt_tokens", "INTEGER"), ("completion_tokens", "INTEGER"),
               ("concurrency", "INTEGER"), ("ttft_p95_s", "REAL"), ("rejected", "INTEGER"), ("capability", "TEXT"),
               ("image_units", "REAL"), ("error", "TEXT")]

    def __init__(self, path: str = ":memory:"):
        self.db = sqlite3.connect(path, check_same_thread=False)
        self.db.row_factory = sqlite3.Row
        self._lock = threading.Lock()
        self.db.execute("CREATE TABLE IF NOT EXISTS runs (id INTEGER PRIMARY KEY AUTOINCREMENT)")
        have = {r["name"] for r in self.db.execute("PRAGMA table_info(runs)")}
        for name, typ in self.COLUMNS:  # add-if-missing: older databases keep their rows
            if name not in have:
                self.db.execute(f"ALTER TABLE runs ADD COLUMN {name} {typ}")
        self.db.commit()

    def insert(self, **row):
        cols = [c for c, _ in self.COLUMNS if c in row]
        with self._lock:
            self.db.execute(f"INSERT INTO runs ({', '.join(cols)}) VALUES ({', '.join('?' * len(cols))})",
                            [row[c] for c in cols])
            self.db.commit()

    def runs(self, limit: int = 100) -> list[dict]:
        return [dict(r) for r in self.db.execute("SELECT * FROM runs ORDER BY id DESC LIMIT ?", (limit,))]

    def series(self, model: str, scenario: str) -> list[dict]:
        return [dict(r) for r in self.db.execute(
            "SELECT ts, version, ttft_s, decode_tps, total_s FROM runs WHERE model = ? AND scenario = ? AND error IS NULL "
            "ORDER BY ts", (model, scenario))]

    def summary(self) -> list[dict]:
        groups: dict[tuple, list] = {}
        for r in self.db.execute("SELECT target, version, model, scenario, ttft_s, decode_tps, total_s FROM runs "
                                 "WHERE error IS NULL"):
            groups.setdefault((r["target"], r["version"], r["model"], r["scenario"]), []).append(r)
        out = []
        for (tgt, ver, model, sc), rows in sorted(groups.items(), key=lambda kv: tuple(str(x) for x in kv[0])):
            med = lambda k: statistics.median(v for v in (x[k] for x in rows) if v is not None) \
                if any(x[k] is not None for x in rows) else None  # noqa: E731
            out.append({"target": tgt, "version": ver, "model": model, "scenario": sc, "runs": len(rows),
                        "ttft_s": med("ttft_s"), "decode_tps": med("decode_tps"), "total_s": med("total_s")})
        return out


@dataclass
class Target:
    name: str
    endpoint: str


@dataclass
class BenchDaemon:
    targets: list[Target]
    store: Store
    scenarios: list[Scenario] = field(default_factory=lambda: list(DEFAULT_SCENARIOS))
    max_tokens: int = 128
    transport: object = None

    async def cycle(self):
        async with httpx.AsyncClient(timeout=600.0, transport=self.transport) as client:
            for t in self.targets:
                try:
                    ver = (await client.get(t.endpoint + "/version")).json().get("git_sha", "unknown")
                    models = (await client.get(t.endpoint + "/v1/models")).json().get("data", [])
                except Exception as e:
                    self.store.insert(ts=time.time(), target=t.name, endpoint=t.endpoint, error=f"discovery: {e}")
                    continue
                for m in models:
                    caps = m.get("capabilities") or ["text"]
                    for sc in self.scenarios:
                        if not sc.applies_to(caps):
                            continue
                        row = dict(ts=time.time(), target=t.name, endpoint=t.endpoint, version=ver, model=m["id"],
                                   scenario=sc.id, prompt_size=sc.prompt_tokens)
                        try:
                            res = await run_scenario(client, t.endpoint, m["id"], sc, self.max_tokens)
                            row.update({k: v for k, v in res.__dict__.items()})
                        except Exception as e:
                            row["error"] = repr(e)[:500]
                        self.store.insert(**row)

    async def run_forever(self, interval_s: float):
        while True:
            await self.cycle()
            await asyncio.sleep(interval_s)


def create_bench_api(store: Store) -> FastAPI:
    app = FastAPI(title="helexa-b200 bench")

    @app.get("/api/health")
    async def health():
        return {"status": "ok", "runs": store.db.execute("SELECT COUNT(*) FROM runs").fetchone()[0]}

    @app.get("/api/summary")
    async def summary():
        return {"summary": store.summary()}

    @app.get("/api/series")
    async def series(model: str, scenario: str):
        return {"model": model, "scenario": scenario, "points": store.series(model, scenario)}

    @app.get("/api/runs")
    async def runs(limit: int = 100):
        return {"runs": store.runs(limit)}

    return app


def main(argv=None):
    import argparse

    import uvicorn
    ap = argparse.ArgumentParser(description="continuous benchmark daemon")
    ap.add_argument("--target", action="append", required=True, help="name=http://host:port (repeatable)")
    ap.add_argument("--db", default="helexa-bench.sqlite")
    ap.add_argument("--interval", type=float, default=3600.0)
    ap.add_argument("--port", type=int, default=8099)
    a = ap.parse_args(argv)
    store = Store(a.db)
    d = BenchDaemon([Target(*t.split("=", 1)) for t in a.target], store)
    app = create_bench_api(store)

    @app.on_event("startup")
    async def _start():
        app.state.loop_task = asyncio.create_task(d.run_forever(a.interval))

    uvicorn.run(app, host="0.0.0.0", port=a.port)


if __name__ == "__main__":
    main()
