"""Logging and tracing: structured log lines, timed spans, NVTX ranges.

The reference instruments its node with `tracing` spans and an env-filter log level
(`RUST_LOG`, main.rs / engine.rs). Here:

  * `setup_logging()` configures the `helexa` logger from `HELEXA_LOG` (level, default
    INFO) and `HELEXA_LOG_FORMAT` (`json` for one JSON object per line, else text);
  * `span(name, **fields)` times a block, logs it at DEBUG (or INFO when `slow_ms` is
    exceeded) with its fields, and -- with `HELEXA_NVTX=1` on a CUDA host -- brackets it
    in an NVTX range so a profiler timeline shows engine phases next to the kernels;
  * `request_span(...)` logs one INFO line per finished request (id, principal, model,
    prompt / cached / completion tokens, prefill / decode milliseconds, finish reason).
"""
from __future__ import annotations

import json
import logging
import os
import time
from contextlib import contextmanager

LOG = logging.getLogger("helexa")
_NVTX = os.environ.get("HELEXA_NVTX") == "1"


class _JsonFormatter(logging.Formatter):
    def format(self, record: logging.LogRecord) -> str:
        out = {"ts": round(record.created, 3), "level": record.levelname.lower(), "logger": record.name,
               "msg": record.getMessage()}
        fields = getattr(record, "fields", None)
        if fields:
            out.update(fields)
        return json.dumps(out, default=str)


def setup_logging(level: str | None = None, fmt: str | None = None) -> logging.Logger:
    level = (level or os.environ.get("HELEXA_LOG", "INFO")).upper()
    fmt = fmt or os.environ.get("HELEXA_LOG_FORMAT", "text")
    h = logging.StreamHandler()
    h.setFormatter(_JsonFormatter() if fmt == "json" else
                   logging.Formatter("%(asctime)s %(levelname)s %(name)s %(message)s"))
    LOG.handlers[:] = [h]
    LOG.setLevel(getattr(logging, level, logging.INFO))
    LOG.propagate = False
    return LOG


def _nvtx(push: bool, name: str = ""):
    if not _NVTX:
        return
    try:
        import torch
        if torch.cuda.is_available():
            if push:
                torch.cuda.nvtx.range_push(name)
            else:
                torch.cuda.nvtx.range_pop()
    except Exception:
        pass


@contextmanager
def span(name: str, slow_ms: float | None = None, **fields):
    """Time a block; log it (DEBUG, or INFO past `slow_ms`) with its fields."""
    _nvtx(True, name)
    t0 = time.perf_counter()
    try:
        yield fields
    finally:
        ms = (time.perf_counter() - t0) * 1e3
        _nvtx(False)
        lvl = logging.INFO if slow_ms is not None and ms > slow_ms else logging.DEBUG
        if LOG.isEnabledFor(lvl):
            LOG.log(lvl, f"span {name} {ms:.2f} ms", extra={"fields": {"span": name, "ms": round(ms, 3), **fields}})


def request_span(rid: str, model: str, principal: str | None, prompt_tokens: int, cached_tokens: int,
                 completion_tokens: int, prefill_ms: float, decode_ms: float, finish: str) -> dict:
    fields = {"request_id": rid, "model": model, "principal": principal or "anonymous",
              "prompt_tokens": prompt_tokens, "cached_tokens": cached_tokens,
              "completion_tokens": completion_tokens, "prefill_ms": round(prefill_ms, 2),
              "decode_ms": round(decode_ms, 2), "finish": finish}
    LOG.info(f"request {rid} {finish} {completion_tokens} tokens", extra={"fields": fields})
    return fields
