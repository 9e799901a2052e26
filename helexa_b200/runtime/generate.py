"""Single-request generation on one model (the public `generate` call).

`Generator.generate` is the end-to-end path a user calls: it copies the prompt from
pinned host memory, prefills (chunked, like the reference's 512-token windows in
harness/candle.rs:1638-1648, but with a configurable window), then replays a
captured multi-step decode graph and reads the produced tokens back. Stop
conditions (EOS, max tokens) are checked once per replayed graph chunk; tokens
produced past a stop are discarded.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch


@dataclass
class GenerateResult:
    tokens: list[int]
    prompt_tokens: int
    ttft_s: float
    decode_s: float
    finish_reason: str
    timings: dict = field(default_factory=dict)

    @property
    def decode_tok_s(self) -> float:
        n = max(0, len(self.tokens) - 1)
        return n / self.decode_s if self.decode_s > 0 else 0.0


class Generator:
    """Drives a FastModel for one slot at a time (bs=1 latency path)."""

    def __init__(self, model, slot: int = 0, graph_steps: int = 16, prefill_chunk: int = 8192):
        self.m = model
        self.slot = slot
        self.graph_steps = graph_steps
        self.prefill_chunk = prefill_chunk
        self.nb = None
        self._pinned_out = torch.empty(model.buffers(1).out_tokens.shape[1], dtype=torch.int32, pin_memory=True)

    def prefill(self, prompt_dev: torch.Tensor, p0: int = 0) -> torch.Tensor:
        logits = None
        for s in range(0, prompt_dev.shape[0], self.prefill_chunk):
            logits = self.m.prefill(self.slot, prompt_dev[s:s + self.prefill_chunk], p0 + s)
        return logits

    @torch.no_grad()
    def generate(self, prompt: torch.Tensor | list[int], max_new_tokens: int, eos_ids=(), ignore_eos=False,
                 p0: int = 0) -> GenerateResult:
        m = self.m
        dev = m.device
        if not isinstance(prompt, torch.Tensor):
            prompt = torch.tensor(prompt, dtype=torch.int32)
        if not prompt.is_pinned():
            prompt = prompt.to(torch.int32).pin_memory()
        stream = torch.cuda.current_stream(dev)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        t0 = time.perf_counter()
        ev[0].record(stream)
        prompt_dev = prompt.to(dev, non_blocking=True)
        logits = self.prefill(prompt_dev, p0)
        nb = m.capture(1, steps=self.graph_steps)
        nb.slots.fill_(self.slot)
        nb.tok.copy_(torch.argmax(logits).to(torch.int32).reshape(1))
        nb.step.zero_()
        ev[1].record(stream)
        first = int(nb.tok[0])  # D2H of the first token (TTFT point)
        ttft = time.perf_counter() - t0
        out = [first]
        finish = "length"
        eos = set(eos_ids)
        if not ignore_eos and first in eos:
            m.check_errors()
            return GenerateResult(out, prompt.numel(), ttft, 0.0, "stop")
        produced = 0
        t1 = time.perf_counter()
        while len(out) < max_new_tokens:
            m.replay(nb)
            produced += self.graph_steps
            cap = nb.out_tokens.shape[1]
            n = self.graph_steps
            start = (produced - n) % cap
            self._pinned_out[:n].copy_(nb.out_tokens[0, start:start + n], non_blocking=True)
            stream.synchronize()
            new = self._pinned_out[:n].tolist()
            stop = False
            for t in new:
                if len(out) >= max_new_tokens:
                    break
                out.append(t)
                if not ignore_eos and t in eos:
                    finish, stop = "stop", True
                    break
            if stop:
                break
        ev[2].record(stream)
        ev[2].synchronize()
        decode_s = time.perf_counter() - t1
        m.check_errors()  # tokens produced after a timed-out wait are not valid
        # The slot's state has advanced over the whole last graph chunk, including any
        # tokens discarded after a stop; callers that continue a sequence restore a
        # prefix snapshot instead of reusing this state.
        return GenerateResult(out, prompt.numel(), ttft, decode_s, finish,
                              timings={"prefill_ms_dev": ev[0].elapsed_time(ev[1]),
                                       "decode_ms_dev": ev[1].elapsed_time(ev[2])})
