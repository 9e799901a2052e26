"""Command line: run a node, run the gateway, print fleet status.

  python -m helexa_b200.cli node   [--host H] [--port P] [--config node.toml]
  python -m helexa_b200.cli serve  [--config cortex.toml]
  python -m helexa_b200.cli status [--endpoint http://localhost:31313]
  python -m helexa_b200.cli router   --config router.toml [--port 8088]
  python -m helexa_b200.cli tools    [--port 8889]
  python -m helexa_b200.cli upstream [--db ledger.sqlite] [--operator-token T=op] [--port 8090]
  python -m helexa_b200.cli bench    --target name=http://host:port [--db bench.sqlite]
  python -m helexa_b200.cli portal   [--db portal.sqlite] [--ledger-db ledger.sqlite] [--port 8091]
  python -m helexa_b200.cli acp      [--base-url http://127.0.0.1:31313/v1] [--model M]

`serve` and `status` are the reference's `cortex serve|status` (cortex-cli/src/main.rs:
15-111). The gateway config is TOML:

  [gateway]
  listen = "0.0.0.0:31313"
  poll_interval_s = 10
  require_auth = false

  [[neurons]]                       # one per node
  name = "gpu-box-1"
  url = "http://10.0.0.5:13131"

  [[models]]                        # catalogue entries (CatalogueEntry fields)
  model_id = "qwen3-8b"
  source = "preset:qwen3-8b"
  aliases = ["fast"]
  tensor_parallel = 2

  [auth.keys]                       # bearer key -> principal
  "sk-abc" = "acct-1"

  [entitlements]                    # principal -> models it may use
  "acct-1" = ["qwen3-8b"]

  [budgets."acct-1"]                # token cap; window_s = 0 is a hard balance
  hard_cap = 1000000
  window_s = 0

`HELEXA_`-prefixed environment variables override keys (`__` separates levels).
"""
from __future__ import annotations

import argparse
import json
import sys


def _gateway_from_config(cfg: dict):
    from .gateway.app import create_gateway
    from .gateway.budget import Cap
    from .gateway.core import Catalogue, CatalogueEntry, NodeState

    cat = Catalogue()
    for m in cfg.get("models", []):
        cat.add(CatalogueEntry(**{k: v for k, v in m.items() if k in CatalogueEntry.__dataclass_fields__}))
    nodes = [NodeState(n["name"], n["url"].rstrip("/")) for n in cfg.get("neurons", [])]
    if not nodes:
        raise SystemExit("config has no [[neurons]] entries")
    gw = cfg.get("gateway", {})
    keys = cfg.get("auth", {}).get("keys") or None
    ents = {p: set(ms) for p, ms in (cfg.get("entitlements") or {}).items()} or None
    budgets = {p: Cap(b.get("hard_cap"), int(b.get("window_s", 0))) for p, b in (cfg.get("budgets") or {}).items()}
    return create_gateway(cat, nodes, api_keys=keys, require_auth=bool(gw.get("require_auth", False)),
                          poll_interval_s=float(gw.get("poll_interval_s", 10.0)), entitlements=ents,
                          budgets=budgets or None)


def _listen(s: str) -> tuple[str, int]:
    host, _, port = s.rpartition(":")
    return host or "0.0.0.0", int(port)


def status_report(endpoint: str, get=None) -> str:
    """Fleet health and the models with their node placements, as printed by `status`."""
    if get is None:
        import httpx

        def get(url):
            r = httpx.get(url, timeout=10.0)
            r.raise_for_status()
            return r.json()
    endpoint = endpoint.rstrip("/")
    health = get(endpoint + "/health")
    models = get(endpoint + "/v1/models")
    lines = ["Fleet health: " + json.dumps(health, indent=2, sort_keys=True), "", "Models:"]
    for m in models.get("data", []):
        where = ", ".join(f"{n}(loaded)" for n in m.get("loaded_on") or []) or "-"
        lim = m.get("limit") or {}
        ctx = f"ctx={lim['context']}" if lim.get("context") else ""
        lines.append(f"  {m.get('id', '?'):40} {where} {ctx}".rstrip())
    return "\n".join(lines)


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(prog="helexa", description="helexa-b200 serving engine")
    sub = ap.add_subparsers(dest="cmd", required=True)
    n = sub.add_parser("node", help="run a node daemon (the serving engine)")
    n.add_argument("--host", default="127.0.0.1")
    n.add_argument("--port", type=int, default=13131)
    n.add_argument("--config")
    s = sub.add_parser("serve", help="run the gateway in front of a fleet of nodes")
    s.add_argument("-c", "--config", default="cortex.toml")
    st = sub.add_parser("status", help="print fleet health and model placements")
    st.add_argument("-e", "--endpoint", default="http://localhost:31313")
    r = sub.add_parser("router", help="run the federation router in front of several gateways")
    r.add_argument("--config", required=True)
    r.add_argument("--host", default="0.0.0.0")
    r.add_argument("--port", type=int, default=8088)
    t = sub.add_parser("tools", help="run the SSRF-guarded fetch tool service")
    t.add_argument("--host", default="127.0.0.1")
    t.add_argument("--port", type=int, default=8889)
    u = sub.add_parser("upstream", help="run the account ledger service")
    u.add_argument("--db", default="helexa-ledger.sqlite")
    u.add_argument("--operator-token", action="append", default=[], help="TOKEN=operator (repeatable)")
    u.add_argument("--signup-allocation", type=int, default=0)
    u.add_argument("--host", default="127.0.0.1")
    u.add_argument("--port", type=int, default=8090)
    b = sub.add_parser("bench", help="run the continuous benchmark daemon")
    b.add_argument("--target", action="append", required=True, help="name=http://host:port (repeatable)")
    b.add_argument("--db", default="helexa-bench.sqlite")
    b.add_argument("--interval", type=float, default=3600.0)
    b.add_argument("--port", type=int, default=8099)
    po = sub.add_parser("portal", help="run the confidential document portal")
    po.add_argument("--db", default="helexa-portal.sqlite")
    po.add_argument("--ledger-db", default="helexa-ledger.sqlite")
    po.add_argument("--host", default="127.0.0.1")
    po.add_argument("--port", type=int, default=8091)
    a = sub.add_parser("acp", help="run the ACP editor agent on stdin / stdout")
    a.add_argument("--base-url", default="http://127.0.0.1:31313/v1")
    a.add_argument("--model", default="default")
    a.add_argument("--api-key")
    args = ap.parse_args(argv)
    if args.cmd in ("router", "tools", "upstream"):
        import uvicorn
        if args.cmd == "router":
            from .mesh.router import RouterConfig, create_router
            app = create_router(RouterConfig.load(args.config))
        elif args.cmd == "tools":
            from .mesh.tools import create_tools_app
            app = create_tools_app()
        else:
            from .mesh.upstream import UpstreamConfig, create_upstream
            toks = dict(x.split("=", 1) for x in args.operator_token)
            app = create_upstream(UpstreamConfig(db_path=args.db, operator_tokens=toks,
                                                 signup_allocation=args.signup_allocation))
        uvicorn.run(app, host=args.host, port=args.port)
        return 0
    if args.cmd == "portal":
        import uvicorn

        from .mesh.portal import Portal, create_portal
        from .mesh.upstream import Ledger
        uvicorn.run(create_portal(Portal(Ledger(args.ledger_db), args.db)), host=args.host, port=args.port)
        return 0
    if args.cmd == "bench":
        from .mesh.benchd import main as bench_main
        argv2 = sum((["--target", x] for x in args.target), []) + ["--db", args.db, "--interval",
                                                                   str(args.interval), "--port", str(args.port)]
        bench_main(argv2)
        return 0
    if args.cmd == "acp":
        from .mesh.acp import main as acp_main
        acp_main(["--base-url", args.base_url, "--model", args.model] +
                 (["--api-key", args.api_key] if args.api_key else []))
        return 0
    if args.cmd == "node":
        from .server.app import main as node_main
        sys.argv = [sys.argv[0], "--host", args.host, "--port", str(args.port)] + \
            (["--config", args.config] if args.config else [])
        node_main()
        return 0
    if args.cmd == "serve":
        import uvicorn

        from .config.settings import load_settings
        cfg = load_settings(args.config)
        app = _gateway_from_config(cfg)
        host, port = _listen(cfg.get("gateway", {}).get("listen", "0.0.0.0:31313"))
        uvicorn.run(app, host=host, port=port)
        return 0
    print(status_report(args.endpoint))
    return 0


if __name__ == "__main__":
    sys.exit(main())
