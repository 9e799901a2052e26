"""Per-model admission control: bounded seats, bounded queue, bounded waits.

Semantics follow harness/admission.rs:1-830:
  * at most `max_in_flight` running requests and `max_queue_depth` waiters; a full
    queue or a wait past `max_wait_s` is refused immediately (429/503 + Retry-After)
    instead of stalling;
  * fair share: an identified principal may hold at most `max_per_principal`
    queued+running requests;
  * anonymous requests (no principal) only use leftover capacity: they never take a
    seat while an identified request waits, they hold at most `anon_max_in_flight`
    seats (default: all but one) and `anon_max_pending` queue places;
  * KV budget: a request may reserve MiB of KV cache; a reservation larger than the
    whole budget is refused permanently (`kv_unservable`), otherwise it waits up to
    `kv_max_wait_s` (`kv_timeout`);
  * `close()` refuses everything new and wakes every waiter (shutdown).

Pure asyncio, no device work; counters are readable without blocking for /health.
"""
from __future__ import annotations

import asyncio
import time
from dataclasses import dataclass, field


@dataclass
class AdmissionConfig:
    max_in_flight: int = 1
    max_queue_depth: int = 8
    max_wait_s: float = 30.0
    max_per_principal: int = 0          # 0 = unlimited
    anon_max_in_flight: int | None = None
    anon_max_pending: int | None = None
    kv_max_wait_s: float = 120.0
    retry_after_s: int = 5


class AdmissionRejection(Exception):
    """Refusal with a reason; `status` is the HTTP status, `retry_after` seconds."""

    STATUS = {"queue_full": 503, "timeout": 503, "per_principal": 429, "anon_yield": 503,
              "kv_timeout": 503, "kv_unservable": 413, "closed": 503}

    def __init__(self, reason: str, retry_after: int = 0, required_mb: int = 0, budget_mb: int = 0):
        self.reason = reason
        self.retry_after = retry_after
        self.required_mb = required_mb
        self.budget_mb = budget_mb
        super().__init__(f"admission rejected: {reason}")

    @property
    def status(self) -> int:
        return self.STATUS.get(self.reason, 503)


@dataclass
class RejectionCounts:
    queue_full: int = 0
    timeout: int = 0
    per_principal: int = 0
    anon_yield: int = 0
    kv_timeout: int = 0
    kv_unservable: int = 0
    closed: int = 0


@dataclass
class _State:
    pending: int = 0
    running: int = 0
    per_principal: dict = field(default_factory=dict)
    anon_pending: int = 0
    anon_running: int = 0
    identified_waiting: int = 0
    kv_used_mb: int = 0


class AdmissionPermit:
    def __init__(self, ctl: "AdmissionController", principal: str | None, kv_mb: int):
        self._ctl = ctl
        self.principal = principal
        self.kv_mb = kv_mb
        self._released = False

    def release(self):
        if not self._released:
            self._released = True
            self._ctl._release(self)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.release()

    async def __aenter__(self):
        return self

    async def __aexit__(self, *exc):
        self.release()


class AdmissionController:
    def __init__(self, cfg: AdmissionConfig | None = None):
        self.cfg = cfg or AdmissionConfig()
        c = self.cfg
        self.anon_max_in_flight = (max(c.max_in_flight - 1, 1 if c.max_in_flight == 1 else 0)
                                   if c.anon_max_in_flight is None else min(c.anon_max_in_flight, c.max_in_flight))
        max_pending = c.max_in_flight + c.max_queue_depth
        self.anon_max_pending = (max_pending - 1 if c.anon_max_pending is None and max_pending > 1 else
                                 (c.anon_max_pending if c.anon_max_pending is not None else max_pending))
        self.anon_max_pending = min(self.anon_max_pending, max_pending)
        self._st = _State()
        self._cond: asyncio.Condition | None = None
        self._closed = False
        self.kv_budget_mb = 0
        self.rejections = RejectionCounts()

    def _condition(self) -> asyncio.Condition:
        if self._cond is None:
            self._cond = asyncio.Condition()
        return self._cond

    # ---- introspection ----------------------------------------------------
    @property
    def in_flight(self) -> int:
        return self._st.running

    @property
    def queue_depth(self) -> int:
        return self._st.pending - self._st.running

    def kv_available_mb(self) -> int:
        return max(0, self.kv_budget_mb - self._st.kv_used_mb)

    def set_kv_budget_mb(self, mb: int):
        self.kv_budget_mb = int(mb)

    def close(self):
        self._closed = True
        if self._cond is not None:
            async def _wake():
                async with self._cond:
                    self._cond.notify_all()
            try:
                asyncio.get_running_loop().create_task(_wake())
            except RuntimeError:
                pass

    # ---- admission -----------------------------------------------------------
    def _reject(self, reason: str, **kw) -> AdmissionRejection:
        setattr(self.rejections, reason, getattr(self.rejections, reason) + 1)
        ra = 0 if reason == "kv_unservable" else self.cfg.retry_after_s
        return AdmissionRejection(reason, ra, **kw)

    async def enter(self, principal: str | None = None, kv_mb: int = 0) -> AdmissionPermit:
        c, st = self.cfg, self._st
        if self._closed:
            raise self._reject("closed")
        anon = principal is None
        if st.pending >= c.max_in_flight + c.max_queue_depth:
            raise self._reject("queue_full")
        if not anon and c.max_per_principal and st.per_principal.get(principal, 0) >= c.max_per_principal:
            raise self._reject("per_principal")
        if anon and (self.anon_max_in_flight == 0 or st.anon_pending >= self.anon_max_pending):
            raise self._reject("anon_yield")
        if kv_mb and self.kv_budget_mb and kv_mb > self.kv_budget_mb:
            raise self._reject("kv_unservable", required_mb=kv_mb, budget_mb=self.kv_budget_mb)
        # reserve a place in line
        st.pending += 1
        if anon:
            st.anon_pending += 1
        else:
            st.per_principal[principal] = st.per_principal.get(principal, 0) + 1
            st.identified_waiting += 1
        cond = self._condition()
        deadline = time.monotonic() + c.max_wait_s
        kv_deadline = time.monotonic() + c.kv_max_wait_s
        admitted = False
        try:
            async with cond:
                while True:
                    if self._closed:
                        raise self._reject("closed")
                    seat_free = st.running < c.max_in_flight
                    kv_ok = (not kv_mb or not self.kv_budget_mb or st.kv_used_mb + kv_mb <= self.kv_budget_mb)
                    if anon:
                        ok = seat_free and st.identified_waiting == 0 and st.anon_running < self.anon_max_in_flight
                    else:
                        ok = seat_free
                    if ok and kv_ok:
                        st.running += 1
                        st.kv_used_mb += kv_mb
                        if anon:
                            st.anon_running += 1
                        else:
                            st.identified_waiting -= 1
                        admitted = True
                        return AdmissionPermit(self, principal, kv_mb)
                    now = time.monotonic()
                    if ok and not kv_ok:
                        limit = kv_deadline
                        why = "kv_timeout"
                    else:
                        limit = deadline
                        why = "anon_yield" if anon and seat_free else "timeout"
                    if now >= limit:
                        raise self._reject(why, required_mb=kv_mb, budget_mb=self.kv_budget_mb) \
                            if why == "kv_timeout" else self._reject(why)
                    try:
                        await asyncio.wait_for(cond.wait(), timeout=limit - now)
                    except asyncio.TimeoutError:
                        pass
        finally:
            if not admitted:
                self._unreserve(principal)
                await self._notify()

    def _unreserve(self, principal: str | None):
        st = self._st
        st.pending -= 1
        if principal is None:
            st.anon_pending -= 1
        else:
            st.per_principal[principal] -= 1
            if not st.per_principal[principal]:
                del st.per_principal[principal]
            st.identified_waiting -= 1

    async def _notify(self):
        cond = self._condition()
        async with cond:
            cond.notify_all()

    def _release(self, permit: AdmissionPermit):
        st = self._st
        st.running -= 1
        st.pending -= 1
        st.kv_used_mb -= permit.kv_mb
        if permit.principal is None:
            st.anon_running -= 1
            st.anon_pending -= 1
        else:
            st.per_principal[permit.principal] -= 1
            if not st.per_principal[permit.principal]:
                del st.per_principal[permit.principal]
        try:
            asyncio.get_running_loop().create_task(self._notify())
        except RuntimeError:
            pass
