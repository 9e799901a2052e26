"""Daemon settings: a TOML/JSON file with `HELEXA_`-prefixed environment overrides
(`__` separates nested keys), like the reference's figment config with `NEURON_`
env overrides (config.rs:450-453).

  HELEXA_PORT=8080                      -> {"port": 8080}
  HELEXA_ADMISSION__MAX_IN_FLIGHT=4     -> {"admission": {"max_in_flight": 4}}
"""
from __future__ import annotations

import json
import os


def _coerce(v: str):
    for fn in (int, float):
        try:
            return fn(v)
        except ValueError:
            pass
    if v.lower() in ("true", "false"):
        return v.lower() == "true"
    try:
        return json.loads(v)
    except ValueError:
        return v


def load_settings(path: str | None = None, env: dict | None = None, prefix: str = "HELEXA_") -> dict:
    cfg: dict = {}
    if path:
        with open(path, "rb") as f:
            raw = f.read()
        if path.endswith(".toml"):
            import tomllib
            cfg = tomllib.loads(raw.decode())
        else:
            cfg = json.loads(raw)
    env = os.environ if env is None else env
    for k, v in env.items():
        if not k.startswith(prefix):
            continue
        keys = k[len(prefix):].lower().split("__")
        d = cfg
        for kk in keys[:-1]:
            d = d.setdefault(kk, {})
        d[keys[-1]] = _coerce(v)
    return cfg
