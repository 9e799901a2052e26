"""Sampling parameters and host-side samplers.

Precedence (harness/sampling.rs:1-368): an explicit request field wins, then the
model's `generation_config.json`, then the fallback (temperature 0.7). A repeat
penalty (default 1.1 over the last 64 tokens) divides positive logits and multiplies
negative ones, like the reference's `sample_with_penalty`.

Greedy decoding never leaves the GPU (the arg-max is fused into the lm_head GEMV);
the host sampler here serves non-greedy requests and the CPU reference model.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

import torch

FALLBACK_TEMPERATURE = 0.7
DEFAULT_REPEAT_PENALTY = 1.1
DEFAULT_REPEAT_LAST_N = 64


@dataclass
class GenerationDefaults:
    """Values read from a model directory's generation_config.json."""
    temperature: float | None = None
    top_p: float | None = None
    top_k: int | None = None
    repetition_penalty: float | None = None
    max_new_tokens: int | None = None
    eos_token_ids: list[int] = field(default_factory=list)

    @classmethod
    def from_dir(cls, path: str) -> "GenerationDefaults":
        f = os.path.join(path, "generation_config.json")
        if not os.path.exists(f):
            return cls()
        with open(f) as fh:
            raw = json.load(fh)
        eos = raw.get("eos_token_id")
        eos = [] if eos is None else ([eos] if isinstance(eos, int) else list(eos))
        return cls(temperature=raw.get("temperature"), top_p=raw.get("top_p"), top_k=raw.get("top_k"),
                   repetition_penalty=raw.get("repetition_penalty"), max_new_tokens=raw.get("max_new_tokens"),
                   eos_token_ids=eos)


@dataclass
class SamplingParams:
    temperature: float = FALLBACK_TEMPERATURE
    top_p: float = 1.0
    top_k: int = 0
    repeat_penalty: float = DEFAULT_REPEAT_PENALTY
    repeat_last_n: int = DEFAULT_REPEAT_LAST_N
    seed: int | None = None
    max_tokens: int = 256
    stop_token_ids: list[int] = field(default_factory=list)
    ignore_eos: bool = False

    @property
    def greedy(self) -> bool:
        return self.temperature <= 0.0 and self.repeat_penalty == 1.0

    @classmethod
    def resolve(cls, request: dict, defaults: GenerationDefaults | None = None, max_tokens_default: int = 256,
                eos_ids: list[int] | None = None) -> "SamplingParams":
        d = defaults or GenerationDefaults()

        def pick(name, dname, fallback):
            v = request.get(name)
            if v is not None:
                return v
            dv = getattr(d, dname)
            return dv if dv is not None else fallback

        temp = float(pick("temperature", "temperature", FALLBACK_TEMPERATURE))
        mt = request.get("max_tokens", request.get("max_completion_tokens"))
        stop_ids = list(eos_ids or []) + list(d.eos_token_ids)
        rp = request.get("repeat_penalty", request.get("repetition_penalty"))
        if rp is None:
            rp = d.repetition_penalty if d.repetition_penalty is not None else DEFAULT_REPEAT_PENALTY
        return cls(temperature=temp, top_p=float(pick("top_p", "top_p", 1.0)),
                   top_k=int(pick("top_k", "top_k", 0) or 0), repeat_penalty=float(rp),
                   seed=request.get("seed"), max_tokens=int(mt if mt is not None else
                                                             (d.max_new_tokens or max_tokens_default)),
                   stop_token_ids=sorted(set(stop_ids)), ignore_eos=bool(request.get("ignore_eos", False)))


def apply_repeat_penalty(logits: torch.Tensor, history: list[int], penalty: float, last_n: int) -> torch.Tensor:
    if penalty == 1.0 or not history:
        return logits
    ids = torch.tensor(sorted(set(history[-last_n:])), dtype=torch.long, device=logits.device)
    sel = logits[ids]
    logits = logits.clone()
    logits[ids] = torch.where(sel > 0, sel / penalty, sel * penalty)
    return logits


class HostSampler:
    """Per-request sampler: repeat penalty, temperature, top-k, top-p, seeded."""

    def __init__(self, params: SamplingParams):
        self.p = params
        self.gen = torch.Generator()
        if params.seed is not None:
            self.gen.manual_seed(int(params.seed))
        else:
            self.gen.seed()

    def sample(self, logits: torch.Tensor, history: list[int]) -> int:
        lg = apply_repeat_penalty(logits.float().cpu(), history, self.p.repeat_penalty, self.p.repeat_last_n)
        if self.p.temperature <= 0.0:
            return int(torch.argmax(lg))
        lg = lg / self.p.temperature
        if self.p.top_k and self.p.top_k < lg.numel():
            kth = torch.topk(lg, self.p.top_k).values[-1]
            lg = lg.masked_fill(lg < kth, float("-inf"))
        probs = torch.softmax(lg, -1)
        if self.p.top_p < 1.0:
            sp, si = torch.sort(probs, descending=True)
            cum = torch.cumsum(sp, -1)
            keep = cum - sp < self.p.top_p
            keep[0] = True
            mask = torch.zeros_like(probs, dtype=torch.bool)
            mask[si[keep]] = True
            probs = torch.where(mask, probs, torch.zeros_like(probs))
            probs = probs / probs.sum()
        return int(torch.multinomial(probs, 1, generator=self.gen))
