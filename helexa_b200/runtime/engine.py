"""Continuous-batching inference engine over a model runner.

One worker thread owns the device (like the reference's per-GPU device thread,
harness/device_worker/mod.rs:1-40): requests are queued to it, and it alternates
  * joins: restore the longest cached prefix snapshot (or reset the slot), prefill up
    to the stable cut (one past the last `<|im_start|>`), snapshot there into the
    prefix cache, prefill the rest, sample the first token;
  * decode: one batched step (or a captured multi-step graph for greedy rows) over
    every live sequence, then stop checks (EOS / stop ids / max tokens / cancel).
Token events are pushed to each request's queue as they are produced
(harness/engine.rs:1-1285; the reference's lockstep (B,1) decode rebatches by
extract/assemble, here every live sequence simply keeps its slot).

A fatal device error poisons the engine: every live and queued request receives an
error and later submissions are refused until the model is reloaded
(harness/candle.rs:1478-1535 poison + recovery).
"""
from __future__ import annotations

import itertools
import queue
import threading
import time
from dataclasses import dataclass, field
from typing import Any

import torch

from ..utils.trace import span
from .prefix_cache import PrefixCache, stable_snapshot_cut
from .sampling import HostSampler, SamplingParams


@dataclass
class TokenEvent:
    token_ids: list[int]


@dataclass
class FinishEvent:
    reason: str                 # "stop" | "length" | "cancelled" | "error"
    prompt_tokens: int
    completion_tokens: int
    cached_tokens: int
    prefill_ms: float
    decode_ms: float
    error: str | None = None


@dataclass
class Request:
    prompt: list[int]
    params: SamplingParams
    id: str = ""
    principal: str | None = None
    mm: Any = None          # MultimodalPrompt (runtime/multimodal.py): prefilled from embeddings
    events: "queue.Queue[Any]" = field(default_factory=queue.Queue)
    cancelled: threading.Event = field(default_factory=threading.Event)

    def cancel(self):
        self.cancelled.set()

    def iter_events(self, timeout: float | None = None):
        while True:
            ev = self.events.get(timeout=timeout)
            yield ev
            if isinstance(ev, FinishEvent):
                return


@dataclass
class _Seq:
    req: Request
    slot: int
    history: list[int]
    produced: int = 0
    last: int = 0
    sampler: HostSampler | None = None
    draws: int = 0          # on-device sampler draws so far (seeded reproducibility)
    seed: int = 0
    t_start: float = 0.0
    t_first: float = 0.0
    cached: int = 0


class EngineError(RuntimeError):
    pass


class Engine:
    def __init__(self, runner, prefix_cache: PrefixCache | None = None, im_start_id: int | None = None,
                 max_batch: int = 4, decode_steps: int = 8, snapshot_min_tokens: int = 64):
        self.runner = runner
        self.prefix_cache = prefix_cache
        self.im_start_id = im_start_id
        self.max_batch = min(max_batch, runner.num_slots)
        self.decode_steps = decode_steps
        self.snapshot_min_tokens = snapshot_min_tokens
        self._in: "queue.Queue[Request]" = queue.Queue()
        self._free = list(range(self.runner.num_slots))
        self._live: list[_Seq] = []
        self._stop = threading.Event()
        self.poisoned: str | None = None
        self._ids = itertools.count()
        self._thread = threading.Thread(target=self._loop, name="helexa-engine", daemon=True)
        self.stats = {"requests": 0, "prefill_tokens": 0, "decode_tokens": 0, "prefix_hits": 0}
        self._thread.start()

    # ---- public ------------------------------------------------------------
    def submit(self, prompt: list[int], params: SamplingParams, principal: str | None = None,
               mm=None) -> Request:
        if self.poisoned:
            raise EngineError(f"model poisoned: {self.poisoned}")
        if not prompt:
            raise ValueError("empty prompt")
        if len(prompt) + params.max_tokens + 1 > self.runner.max_len:
            raise ValueError(f"prompt ({len(prompt)}) + max_tokens ({params.max_tokens}) exceeds the context "
                             f"window ({self.runner.max_len})")
        if mm is not None and not hasattr(self.runner, "prefill_mm"):
            raise ValueError("this model's runner cannot prefill image inputs")
        req = Request(prompt=list(prompt), params=params, principal=principal, mm=mm, id=f"req-{next(self._ids)}")
        self._in.put(req)
        return req

    def generate(self, prompt: list[int], params: SamplingParams, mm=None) -> tuple[list[int], FinishEvent]:
        req = self.submit(prompt, params, mm=mm)
        toks: list[int] = []
        for ev in req.iter_events():
            if isinstance(ev, TokenEvent):
                toks.extend(ev.token_ids)
            else:
                return toks, ev
        raise EngineError("stream ended without a finish event")

    @property
    def in_flight(self) -> int:
        return len(self._live)

    @property
    def queue_depth(self) -> int:
        return self._in.qsize()

    def shutdown(self, timeout: float = 10.0):
        self._stop.set()
        self._in.put(None)  # type: ignore[arg-type]
        self._thread.join(timeout)

    # ---- worker ------------------------------------------------------------
    def _loop(self):
        while not self._stop.is_set():
            try:
                self._admit_new()
                if self._live:
                    self._decode_round()
            except Exception as e:  # device fault or bug: poison, fail everything
                self._poison(repr(e))

    def _admit_new(self):
        block = not self._live
        while self._free and len(self._live) < self.max_batch:
            try:
                req = self._in.get(timeout=0.05) if block else self._in.get_nowait()
            except queue.Empty:
                return
            if req is None:
                return
            block = False
            if req.cancelled.is_set():
                req.events.put(FinishEvent("cancelled", len(req.prompt), 0, 0, 0.0, 0.0))
                continue
            try:
                self._join(req)
            except Exception as e:
                req.events.put(FinishEvent("error", len(req.prompt), 0, 0, 0.0, 0.0, repr(e)))
                raise

    def _join(self, req: Request):
        with span("engine.join", slow_ms=5000, request=req.id, prompt_tokens=len(req.prompt)):
            self._join_inner(req)

    def _join_inner(self, req: Request):
        r = self.runner
        slot = self._free.pop()
        t0 = time.perf_counter()
        p0 = 0
        cached = 0
        if req.mm is not None:
            # image prompts: one embedding prefill; the prefix cache is keyed by token ids,
            # which do not identify an image, so it is neither read nor written
            r.reset(slot)
            logits = r.prefill_mm(slot, req.mm)
            self.stats["prefill_tokens"] += len(req.prompt)
            self._start(req, slot, logits, t0, 0)
            return
        snap = self.prefix_cache.longest_match(req.prompt) if self.prefix_cache else None
        if snap is not None:
            r.restore(slot, snap.snapshot)
            p0 = cached = snap.snapshot.length
            self.stats["prefix_hits"] += 1
        else:
            r.reset(slot)
        prompt = req.prompt
        if self.prefix_cache is not None:
            cut = stable_snapshot_cut(prompt, self.im_start_id)
            if cut - p0 >= self.snapshot_min_tokens and cut < len(prompt):
                r.prefill(slot, prompt[p0:cut], p0)
                s = r.snapshot(slot, cut)
                self.prefix_cache.insert(prompt[:cut], s, s.nbytes)
                p0 = cut
        logits = r.prefill(slot, prompt[p0:], p0)
        self.stats["prefill_tokens"] += len(prompt) - cached
        self._start(req, slot, logits, t0, cached)

    def _start(self, req: Request, slot: int, logits, t0: float, cached: int):
        """First token from the prefill logits; the sequence joins the decode batch."""
        seq = _Seq(req=req, slot=slot, history=list(req.prompt), t_start=t0, cached=cached)
        if not req.params.greedy:
            seq.sampler = HostSampler(req.params)
            seq.seed = int(req.params.seed) if req.params.seed is not None else \
                int(torch.randint(0, 2 ** 62, (1,), generator=seq.sampler.gen))
            tok = seq.sampler.sample(logits, seq.history)
        else:
            tok = int(torch.argmax(logits))
        seq.t_first = time.perf_counter()
        self._live.append(seq)
        self._emit(seq, [tok])

    def _emit(self, seq: _Seq, toks: list[int]):
        """Append produced tokens, stopping at EOS / stop ids / max tokens."""
        p = seq.req.params
        out = []
        reason = None
        for t in toks:
            out.append(t)
            seq.produced += 1
            seq.history.append(t)
            seq.last = t
            if not p.ignore_eos and t in p.stop_token_ids:
                reason = "stop"
                break
            if seq.produced >= p.max_tokens:
                reason = "length"
                break
        if out:
            seq.req.events.put(TokenEvent(out))
            self.stats["decode_tokens"] += len(out)
        if reason is None and seq.req.cancelled.is_set():
            reason = "cancelled"
        if reason is not None:
            self._finish(seq, reason)

    def _finish(self, seq: _Seq, reason: str, error: str | None = None):
        now = time.perf_counter()
        seq.req.events.put(FinishEvent(reason, len(seq.req.prompt), seq.produced, seq.cached,
                                       (seq.t_first - seq.t_start) * 1e3, (now - seq.t_first) * 1e3, error))
        if seq in self._live:
            self._live.remove(seq)
            self._free.append(seq.slot)
        self.stats["requests"] += 1

    def _decode_round(self):
        with span("engine.decode_round", slow_ms=1000, live=len(self._live)):
            self._decode_round_inner()

    def _decode_round_inner(self):
        r = self.runner
        greedy = [s for s in self._live if s.sampler is None]
        sampled = [s for s in self._live if s.sampler is not None]
        if greedy:
            if getattr(r, "greedy_on_device", False):
                left = min(s.req.params.max_tokens - s.produced for s in greedy)
                steps = max(1, min(self.decode_steps, left))
                outs = r.decode([s.slot for s in greedy], [s.last for s in greedy], steps)
            else:
                outs = r.decode([s.slot for s in greedy], [s.last for s in greedy], 1)
            for s, o in zip(greedy, outs):
                self._emit(s, o)
        if sampled and getattr(r, "sample_on_device", False):
            # temperature / top-k / top-p / repeat penalty on the device, several steps
            # per replayed graph (no per-token logits copy to the host)
            left = min(s.req.params.max_tokens - s.produced for s in sampled)
            steps = max(1, min(self.decode_steps, left))
            outs = r.decode_sampled([s.slot for s in sampled], [s.last for s in sampled], steps,
                                    [s.req.params for s in sampled], [s.history for s in sampled],
                                    [s.draws for s in sampled], [s.seed for s in sampled])
            for s, o in zip(sampled, outs):
                s.draws += len(o)
                self._emit(s, o)
        elif sampled:
            lg = r.decode_logits([s.slot for s in sampled], [s.last for s in sampled])
            for s, row in zip(sampled, lg):
                self._emit(s, [s.sampler.sample(row, s.history)])

    def _poison(self, why: str):
        self.poisoned = why
        for s in list(self._live):
            self._finish(s, "error", why)
        while True:
            try:
                req = self._in.get_nowait()
            except queue.Empty:
                break
            if req is not None:
                req.events.put(FinishEvent("error", len(req.prompt), 0, 0, 0.0, 0.0, why))
        self._stop.set()
