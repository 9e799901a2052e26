"""Context-limit derivation from memory and throughput (harness/context_limit.rs:1-447).

The servable context is bounded by (a) the model's position limit, (b) how many tokens
of KV cache fit in the tightest device's free memory after a safety floor, and (c) a
prefill-time budget: at the measured prefill rate (EMA), a prompt must prefill within
`max_prefill_s`. Qwen3-Next's GDN layers hold O(1) state, so only its full-attention
layers count toward KV bytes per token. The same numbers give the admission
controller's KV budget and each request's reservation.
"""
from __future__ import annotations

from dataclasses import dataclass

from ..config import ModelConfig


@dataclass
class ContextProfile:
    kv_bytes_per_token: int        # summed over layers, per sequence, per rank
    state_bytes_per_seq: int       # GDN conv + recurrent state
    max_position: int

    @classmethod
    def from_config(cls, cfg: ModelConfig, tp: int = 1) -> "ContextProfile":
        kv_heads_per_rank = max(1, cfg.num_key_value_heads // tp)
        kv = 2 * cfg.num_full_layers * kv_heads_per_rank * cfg.head_dim * 2
        return cls(kv_bytes_per_token=kv, state_bytes_per_seq=cfg.gdn_state_bytes() // max(1, tp),
                   max_position=cfg.max_position_embeddings)


@dataclass
class DerivedLimit:
    context: int
    input: int
    output: int
    kv_budget_mb: int


def derive_limit(profile: ContextProfile, free_bytes_tightest: int, floor_bytes: int = 1500 << 20,
                 prefill_tok_s: float = 0.0, max_prefill_s: float = 120.0, max_output: int = 32768,
                 concurrent: int = 1) -> DerivedLimit:
    usable = max(0, free_bytes_tightest - floor_bytes - concurrent * profile.state_bytes_per_seq)
    by_mem = usable // max(1, profile.kv_bytes_per_token * concurrent) if profile.kv_bytes_per_token else \
        profile.max_position
    ctx = int(min(profile.max_position, by_mem))
    inp = ctx - 1
    if prefill_tok_s > 0:
        inp = int(min(inp, prefill_tok_s * max_prefill_s))
    return DerivedLimit(context=max(ctx, 0), input=max(inp, 0), output=int(min(max_output, max(ctx - 1, 0))),
                        kv_budget_mb=int(usable >> 20))


def kv_reservation_mb(profile: ContextProfile, prompt_tokens: int, max_tokens: int) -> int:
    """MiB a request reserves against the KV budget while it runs."""
    b = (prompt_tokens + max_tokens) * profile.kv_bytes_per_token + profile.state_bytes_per_seq
    return (b + (1 << 20) - 1) >> 20
