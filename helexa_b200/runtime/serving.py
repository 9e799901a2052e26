"""A loaded, servable model: chat rendering, admission, engine, streamed events.

Request flow (harness/candle.rs:3154-3358 and 7378-7672 in the reference):
render the prompt with the model's chat template (tools, enable_thinking,
chat_template_kwargs) -> tokenize -> validate the prompt cap and context window ->
admission (seat, queue, principal fair-share, KV reservation) -> engine (prefix cache,
prefill, batched decode) -> incremental detokenisation -> reasoning / tool-call
routing -> `InferenceEvent`s (wire/event.rs:38-140).
"""
from __future__ import annotations

import asyncio
import json
import os
import time
import uuid
from dataclasses import dataclass, field

from .admission import AdmissionController, AdmissionRejection
from ..utils.trace import request_span
from .engine import Engine, FinishEvent, TokenEvent
from .sampling import GenerationDefaults, SamplingParams
from .multimodal import request_images
from .tokenizer import IncrementalDetokenizer, StreamParser, parse_tool_call_body


# ---- events -------------------------------------------------------------------
@dataclass
class Start:
    id: str
    model: str
    created: int


@dataclass
class TextDelta:
    text: str


@dataclass
class ReasoningDelta:
    text: str


@dataclass
class ToolCall:
    index: int
    id: str
    name: str
    arguments: str


@dataclass
class Finish:
    reason: str
    prompt_tokens: int
    completion_tokens: int
    reasoning_tokens: int
    cached_tokens: int
    prefill_ms: float
    decode_ms: float
    prefill_tokens: int
    error: str | None = None


class RequestError(Exception):
    """Client error mapped to the OpenAI error envelope (status, code)."""

    def __init__(self, message: str, status: int = 400, code: str = "invalid_request_error"):
        super().__init__(message)
        self.status = status
        self.code = code


@dataclass
class ModelLimits:
    context: int
    input: int
    output: int


@dataclass
class ThroughputEma:
    """Exponential moving averages of prefill and decode rates (context_limit.rs)."""
    alpha: float = 0.2
    prefill_tok_s: float = 0.0
    decode_tok_s: float = 0.0

    def update(self, prefill_tokens: int, prefill_ms: float, decode_tokens: int, decode_ms: float):
        if prefill_ms > 0 and prefill_tokens:
            r = prefill_tokens / (prefill_ms / 1e3)
            self.prefill_tok_s = r if not self.prefill_tok_s else (1 - self.alpha) * self.prefill_tok_s + self.alpha * r
        if decode_ms > 0 and decode_tokens > 1:
            r = (decode_tokens - 1) / (decode_ms / 1e3)
            self.decode_tok_s = r if not self.decode_tok_s else (1 - self.alpha) * self.decode_tok_s + self.alpha * r


@dataclass
class ServedModel:
    model_id: str
    engine: Engine
    tokenizer: object
    config: object
    admission: AdmissionController
    defaults: GenerationDefaults = field(default_factory=GenerationDefaults)
    max_prompt_tokens: int = int(os.environ.get("HELEXA_MAX_PROMPT_TOKENS", "16384"))
    devices: list = field(default_factory=list)
    tensor_parallel: int = 1
    capabilities: list = field(default_factory=lambda: ["chat", "completion"])
    status: str = "loaded"
    spec: dict = field(default_factory=dict)
    ema: ThroughputEma = field(default_factory=ThroughputEma)
    kv_bytes_per_token: int = 0
    # refuse new requests while the tightest device has less free memory than this floor
    # (prefill activations come from the caching allocator); the reference's
    # NEURON_MIN_FREE_VRAM_MB guard
    min_free_vram_mb: int = int(os.environ.get("HELEXA_MIN_FREE_VRAM_MB", "1500"))
    free_vram_mb: object = None  # callable -> MiB free on the tightest device, or None (no check)
    vision: object = None        # VisionFrontend (runtime/multimodal.py) for image inputs, or None

    # prompts must prefill within this many seconds at the measured prefill rate
    max_prefill_s: float = float(os.environ.get("HELEXA_MAX_PREFILL_S", "120"))

    @property
    def limits(self) -> ModelLimits:
        """Context = the KV length the runner was sized for (derived from free device
        memory at load); input additionally bounded by the prompt cap and by the
        prefill-time budget at the EMA prefill rate (harness/context_limit.rs)."""
        ctx = self.engine.runner.max_len
        inp = min(self.max_prompt_tokens, ctx - 1)
        if self.ema.prefill_tok_s > 0:
            inp = max(1, min(inp, int(self.ema.prefill_tok_s * self.max_prefill_s)))
        return ModelLimits(context=ctx, input=inp, output=max(1, ctx - 1))

    # ---- prompt -------------------------------------------------------------
    def render_chat(self, request: dict, include_thinking: bool) -> tuple[list[int], bool]:
        msgs = request.get("messages")
        if not isinstance(msgs, list) or not msgs:
            raise RequestError("'messages' must be a non-empty array")
        kwargs = dict(request.get("chat_template_kwargs") or {})
        enable_thinking = kwargs.pop("enable_thinking", include_thinking)
        text = self.tokenizer.apply_chat_template(msgs, add_generation_prompt=True,
                                                  enable_thinking=enable_thinking,
                                                  tools=request.get("tools"), **kwargs)
        starts_in_think = enable_thinking and text.rstrip().endswith("<think>")
        return self.tokenizer.encode(text), starts_in_think

    def _validate(self, ids: list[int], params: SamplingParams):
        if self.free_vram_mb is not None:
            free = self.free_vram_mb()
            if free is not None and free < self.min_free_vram_mb:
                raise RequestError(f"only {int(free)} MiB of device memory free (floor {self.min_free_vram_mb} MiB)",
                                   503, "insufficient_vram")
        lim = self.limits
        if len(ids) > lim.input:
            raise RequestError(f"prompt has {len(ids)} tokens; this model accepts at most {lim.input}",
                               400, "context_length_exceeded")
        if len(ids) + params.max_tokens + 1 > lim.context:
            params.max_tokens = max(1, lim.context - len(ids) - 1)

    # ---- streaming ------------------------------------------------------------
    async def stream(self, request: dict, principal: str | None = None, include_thinking: bool = False,
                     prompt_ids: list[int] | None = None, start_in_reasoning: bool | None = None):
        if self.status != "loaded":
            raise RequestError(f"model {self.model_id} is {self.status}", 503, "model_unavailable")
        mm = None
        if prompt_ids is None:
            ids, think = self.render_chat(request, include_thinking)
            try:
                uris = request_images(request.get("messages"))
            except ValueError as e:
                raise RequestError(str(e)) from e
            if uris:
                if self.vision is None:
                    raise RequestError(f"model {self.model_id} does not accept image inputs", 400,
                                       "unsupported_content")
                try:
                    mm = await asyncio.to_thread(self.vision.build, ids, uris)
                except ValueError as e:
                    raise RequestError(f"image input: {e}") from e
                ids = mm.tokens
        else:
            ids, think = prompt_ids, False
        if start_in_reasoning is not None:
            think = start_in_reasoning
        params = SamplingParams.resolve(request, self.defaults, eos_ids=self.tokenizer.eos_ids)
        self._validate(ids, params)
        kv_mb = (len(ids) + params.max_tokens) * self.kv_bytes_per_token // (1 << 20)
        permit = await self.admission.enter(principal, kv_mb)
        req = None
        try:
            try:
                req = self.engine.submit(ids, params, principal, mm=mm)
            except ValueError as e:
                raise RequestError(str(e)) from e
            rid = "chatcmpl-" + uuid.uuid4().hex[:24]
            yield Start(rid, self.model_id, int(time.time()))
            detok = IncrementalDetokenizer(self.tokenizer)
            parser = StreamParser(start_in_reasoning=think)
            n_tool = 0
            reasoning_tokens = 0
            while True:
                ev = await asyncio.to_thread(req.events.get)
                if isinstance(ev, TokenEvent):
                    if parser.mode == "reasoning":
                        reasoning_tokens += len(ev.token_ids)
                    text = detok.push(ev.token_ids)
                    for d in parser.feed(text):
                        out = self._route(d, n_tool)
                        if isinstance(out, ToolCall):
                            n_tool += 1
                        yield out
                elif isinstance(ev, FinishEvent):
                    for d in parser.feed("", final=True):
                        out = self._route(d, n_tool)
                        if isinstance(out, ToolCall):
                            n_tool += 1
                        yield out
                    reason = ev.reason
                    if n_tool and reason == "stop":
                        reason = "tool_calls"
                    self.ema.update(len(ids) - ev.cached_tokens, ev.prefill_ms, ev.completion_tokens, ev.decode_ms)
                    request_span(rid, self.model_id, principal, ev.prompt_tokens, ev.cached_tokens,
                                 ev.completion_tokens, ev.prefill_ms, ev.decode_ms, ev.reason)
                    if ev.reason == "error":
                        self.status = "poisoned"
                    yield Finish(reason, ev.prompt_tokens, ev.completion_tokens, reasoning_tokens, ev.cached_tokens,
                                 ev.prefill_ms, ev.decode_ms, len(ids) - ev.cached_tokens, ev.error)
                    return
        except (asyncio.CancelledError, GeneratorExit):
            if req is not None:
                req.cancel()
            raise
        finally:
            permit.release()

    @staticmethod
    def _route(d, index: int):
        if d.kind == "text":
            return TextDelta(d.text)
        if d.kind == "reasoning":
            return ReasoningDelta(d.text)
        name, args = parse_tool_call_body(d.text)
        return ToolCall(index, "call_" + uuid.uuid4().hex[:24], name, json.dumps(args))

    async def complete(self, request: dict, principal: str | None = None, include_thinking: bool = False,
                       prompt_ids: list[int] | None = None):
        """Non-streaming: collect the stream."""
        text, reasoning, tools = [], [], []
        start = fin = None
        async for ev in self.stream(request, principal, include_thinking, prompt_ids):
            if isinstance(ev, Start):
                start = ev
            elif isinstance(ev, TextDelta):
                text.append(ev.text)
            elif isinstance(ev, ReasoningDelta):
                reasoning.append(ev.text)
            elif isinstance(ev, ToolCall):
                tools.append(ev)
            elif isinstance(ev, Finish):
                fin = ev
        return start, "".join(text), "".join(reasoning), tools, fin


__all__ = ["ServedModel", "Start", "TextDelta", "ReasoningDelta", "ToolCall", "Finish", "RequestError",
           "AdmissionRejection", "ModelLimits"]
