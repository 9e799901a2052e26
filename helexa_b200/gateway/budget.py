"""Per-principal token budgets with reserve -> settle accounting.

Before a request is dispatched the gateway reserves its upper-bound cost (prompt
estimate + maximum output) against the principal's hard cap; when the response ends
it settles with the tokens actually used, which releases the unused part. A request
that never reports usage (pre-dispatch failure, dropped stream) releases the whole
reservation. Reservations count against the cap while outstanding, so concurrent
requests can never overshoot it (cortex-core/src/entitlements.rs:44-147,
cortex-gateway/src/metering.rs:1-120).

Two cap windows, as in the reference:
  balance   a hard balance that never resets: exhaustion is `429 insufficient_quota`
            with no Retry-After;
  rolling   a window of `seconds` that resets: exhaustion is `429 rate_limit_exceeded`
            with Retry-After until the window resets.
"""
from __future__ import annotations

import itertools
import json
import threading
import time
from dataclasses import dataclass, field

FALLBACK_MAX_OUTPUT = 4096


class BudgetExceeded(Exception):
    def __init__(self, code: str, message: str, retry_after: int = 0):
        super().__init__(message)
        self.code, self.retry_after = code, retry_after


@dataclass
class Cap:
    hard_cap: int | None            # tokens; None = uncapped
    window_s: int = 0               # 0 = balance (never resets)


@dataclass
class _Account:
    cap: Cap
    spent: int = 0
    reserved: int = 0
    window_start: float = field(default_factory=time.monotonic)


@dataclass
class Reservation:
    id: int
    principal: str
    reserved: int


class BudgetLedger:
    def __init__(self, caps: dict[str, Cap] | None = None, clock=time.monotonic):
        self._acc = {p: _Account(c, window_start=clock()) for p, c in (caps or {}).items()}
        self._ids = itertools.count(1)
        self._mu = threading.Lock()
        self._clock = clock
        self._open: dict[int, Reservation] = {}

    def _roll(self, a: _Account) -> None:
        if a.cap.window_s and self._clock() - a.window_start >= a.cap.window_s:
            a.window_start = self._clock()
            a.spent = 0

    def reserve(self, principal: str | None, tokens: int) -> Reservation | None:
        """Reserve `tokens` for `principal`; None for principals without a cap."""
        if principal is None:
            return None
        with self._mu:
            a = self._acc.get(principal)
            if a is None or a.cap.hard_cap is None:
                return None
            self._roll(a)
            avail = a.cap.hard_cap - a.spent - a.reserved
            if tokens > avail:
                if a.cap.window_s:
                    left = int(a.cap.window_s - (self._clock() - a.window_start)) + 1
                    raise BudgetExceeded("rate_limit_exceeded",
                                         f"rolling-window budget exhausted ({tokens} requested, {max(avail, 0)} "
                                         f"available); resets in {left}s", retry_after=left)
                raise BudgetExceeded("insufficient_quota",
                                     f"hard balance exhausted ({tokens} requested, {max(avail, 0)} available)")
            a.reserved += tokens
            r = Reservation(next(self._ids), principal, tokens)
            self._open[r.id] = r
            return r

    def settle(self, r: Reservation | None, actual: int) -> None:
        """Record `actual` tokens of spend and release the rest of the reservation."""
        if r is None:
            return
        with self._mu:
            if self._open.pop(r.id, None) is None:
                return  # settled or released already: a reservation resolves once
            a = self._acc[r.principal]
            a.reserved -= r.reserved
            self._roll(a)
            a.spent += max(0, actual)

    def release(self, r: Reservation | None) -> None:
        if r is None:
            return
        with self._mu:
            if self._open.pop(r.id, None) is None:
                return
            self._acc[r.principal].reserved -= r.reserved

    def snapshot(self, principal: str) -> dict | None:
        with self._mu:
            a = self._acc.get(principal)
            if a is None:
                return None
            self._roll(a)
            return {"hard_cap": a.cap.hard_cap, "spent": a.spent, "reserved": a.reserved,
                    "window_s": a.cap.window_s}


def estimate_prompt_tokens(body: dict) -> int:
    """Prompt-token estimate at about 4 characters per token over the message text (the
    gateway has no tokenizer; under-counting is the safe side, the node enforces the
    exact limit)."""
    chars = 0
    msgs = body.get("messages")
    if isinstance(msgs, list):
        for m in msgs:
            c = m.get("content") if isinstance(m, dict) else None
            if isinstance(c, str):
                chars += len(c)
            elif isinstance(c, list):
                chars += sum(len(p.get("text", "")) for p in c if isinstance(p, dict))
            chars += 8  # role and template overhead per message
        if isinstance(body.get("system"), str):  # Anthropic system prompt
            chars += len(body["system"])
    elif isinstance(body.get("prompt"), str):
        chars = len(body["prompt"])
    elif isinstance(body.get("input"), str):  # Responses API
        chars = len(body["input"])
    else:
        chars = len(json.dumps(body))
    return max(1, chars // 4)


def reservation_estimate(body: dict, advertised_output: int | None) -> int:
    out = body.get("max_tokens") or body.get("max_completion_tokens") or body.get("max_output_tokens")
    if not isinstance(out, int) or out <= 0:
        out = advertised_output or FALLBACK_MAX_OUTPUT
    return estimate_prompt_tokens(body) + out


class SSEUsage:
    """Incremental SSE reader that keeps the usage a streamed response reports.

    Handles the three wire shapes the node emits: OpenAI chat chunks (top-level
    `usage`), Responses events (`response.usage` on `response.completed`) and Anthropic
    events (`message.usage.input_tokens` on `message_start`, `usage.output_tokens` on
    `message_delta`). Bytes arrive in arbitrary chunks; only complete lines are parsed.
    """

    def __init__(self):
        self._buf = b""
        self.prompt = 0
        self.completion = 0
        self.seen = False

    def feed(self, chunk: bytes) -> None:
        self._buf += chunk
        *lines, self._buf = self._buf.split(b"\n")
        for ln in lines:
            ln = ln.strip()
            if not ln.startswith(b"data:"):
                continue
            payload = ln[5:].strip()
            if not payload or payload == b"[DONE]":
                continue
            try:
                ev = json.loads(payload)
            except json.JSONDecodeError:
                continue
            if isinstance(ev, dict):
                self._take(ev)

    def _take(self, ev: dict) -> None:
        u = ev.get("usage")
        if not isinstance(u, dict) and isinstance(ev.get("response"), dict):
            u = ev["response"].get("usage")
        if not isinstance(u, dict) and isinstance(ev.get("message"), dict):
            u = ev["message"].get("usage")
        if not isinstance(u, dict):
            return
        p = u.get("prompt_tokens", u.get("input_tokens"))
        c = u.get("completion_tokens", u.get("output_tokens"))
        if isinstance(p, int) and p:
            self.prompt = p
        if isinstance(c, int) and (c or not self.completion):
            self.completion = c
        self.seen = True
