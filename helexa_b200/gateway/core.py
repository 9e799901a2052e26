"""Gateway control plane: catalogue, node state, routing, eviction.

Behaviour follows the reference's cortex gateway:
  * catalogue (cortex-core/src/catalogue.rs:77-240): per model an alias list,
    `residency_priority` (pinned models are never evicted), `may_displace`, and a load
    spec (source, tensor_parallel, devices);
  * routing (cortex-gateway/src/router.rs:125-283): resolve alias -> a node where the
    model is loaded and least busy (in-flight + queued from /health; ties break by
    node name) -> if only recovering copies exist, hold and retry -> otherwise
    cold-load on the node with the most free memory, evicting least-recently-used
    displaceable models first (evictor.rs:13-115).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field


@dataclass
class CatalogueEntry:
    model_id: str
    source: str
    aliases: list[str] = field(default_factory=list)
    residency_priority: int = 0       # higher = more resident; >= 100 means pinned
    may_displace: bool = True
    tensor_parallel: int = 1
    memory_mb: int = 0
    load_spec: dict = field(default_factory=dict)
    # advertised price per million tokens (the reference's catalogue cost fields)
    cost_input_per_mtok: float | None = None
    cost_output_per_mtok: float | None = None

    @property
    def pinned(self) -> bool:
        return self.residency_priority >= 100


class Catalogue:
    def __init__(self, entries: list[CatalogueEntry] | None = None):
        self.entries: dict[str, CatalogueEntry] = {}
        self.alias: dict[str, str] = {}
        for e in entries or []:
            self.add(e)

    def add(self, e: CatalogueEntry):
        self.entries[e.model_id] = e
        for a in e.aliases:
            self.alias[a] = e.model_id

    def resolve(self, name: str) -> str:
        return self.alias.get(name, name)

    @classmethod
    def from_toml(cls, path: str) -> "Catalogue":
        import tomllib
        with open(path, "rb") as f:
            raw = tomllib.load(f)
        out = cls()
        for m in raw.get("models", []):
            out.add(CatalogueEntry(**{k: v for k, v in m.items() if k in CatalogueEntry.__dataclass_fields__}))
        return out


@dataclass
class NodeState:
    name: str
    url: str
    healthy: bool = True
    fail_count: int = 0
    models: dict = field(default_factory=dict)       # model_id -> {"status", ...}
    load: dict = field(default_factory=dict)         # model_id -> {"in_flight", "queue_depth"}
    free_mb: int = 0
    last_used: dict = field(default_factory=dict)    # model_id -> monotonic time
    last_poll: float = 0.0

    def busy(self, model_id: str) -> int:
        ld = self.load.get(model_id, {})
        return int(ld.get("in_flight", 0)) + int(ld.get("queue_depth", 0))


class NoRoute(Exception):
    def __init__(self, message: str, status: int = 404, code: str = "model_not_found", retry_after: int = 0):
        super().__init__(message)
        self.status = status
        self.code = code
        self.retry_after = retry_after


@dataclass
class RouteDecision:
    node: NodeState
    model_id: str
    action: str                     # "route" | "cold_load"
    evict: list[str] = field(default_factory=list)


class Router:
    def __init__(self, catalogue: Catalogue, nodes: list[NodeState], unhealthy_after: int = 3):
        self.cat = catalogue
        self.nodes = {n.name: n for n in nodes}
        self.unhealthy_after = unhealthy_after

    # ---- poller input ------------------------------------------------------
    def observe(self, node: str, models: list[dict] | None, health: dict | None, free_mb: int | None = None):
        n = self.nodes[node]
        if models is None:
            n.fail_count += 1
            if n.fail_count >= self.unhealthy_after:   # debounced unhealthy marking
                n.healthy = False
            return
        n.fail_count = 0
        n.healthy = True
        n.models = {m["id"]: m for m in models}
        if health:
            n.load = health.get("models", {})
        if free_mb is not None:
            n.free_mb = free_mb
        n.last_poll = time.monotonic()

    # ---- decision ------------------------------------------------------------
    def route(self, requested: str) -> RouteDecision:
        mid = self.cat.resolve(requested)
        healthy = [n for n in self.nodes.values() if n.healthy]
        loaded = [n for n in healthy if n.models.get(mid, {}).get("status") == "loaded"]
        if loaded:
            best = min(loaded, key=lambda n: (n.busy(mid), n.name))
            best.last_used[mid] = time.monotonic()
            return RouteDecision(best, mid, "route")
        if any(n.models.get(mid, {}).get("status") in ("recovering", "loading") for n in healthy):
            raise NoRoute(f"{mid} is recovering", 503, "model_recovering", retry_after=5)
        entry = self.cat.entries.get(mid)
        if entry is None:
            raise NoRoute(f"model {requested!r} is not in the catalogue", 404, "model_not_found")
        if not healthy:
            raise NoRoute("no healthy nodes", 503, "no_capacity", retry_after=10)
        need = entry.memory_mb
        # prefer a node that fits without eviction, then one that fits after evicting
        # displaceable models (LRU first), else the node with the most free memory
        fits = [n for n in healthy if n.free_mb >= need]
        if fits:
            return RouteDecision(max(fits, key=lambda n: (n.free_mb, n.name)), mid, "cold_load")
        best_plan = None
        for n in healthy:
            victims, freed = [], n.free_mb
            cands = []
            for vid, v in n.models.items():
                ve = self.cat.entries.get(vid)
                if v.get("status") != "loaded" or (ve is not None and (ve.pinned or not entry.may_displace)):
                    continue
                if n.busy(vid):
                    continue
                cands.append((n.last_used.get(vid, 0.0), vid, (ve.memory_mb if ve else 0)))
            for _, vid, mb in sorted(cands):
                if freed >= need:
                    break
                victims.append(vid)
                freed += mb
            if freed >= need and (best_plan is None or len(victims) < len(best_plan[1])):
                best_plan = (n, victims)
        if best_plan is not None:
            return RouteDecision(best_plan[0], mid, "cold_load", evict=best_plan[1])
        n = max(healthy, key=lambda n: (n.free_mb, n.name))
        return RouteDecision(n, mid, "cold_load")
