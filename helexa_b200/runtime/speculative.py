"""Speculative decoding acceptance (greedy), as in harness/speculative.rs:1-234.

A draft proposes k tokens; the target model scores the prompt tail plus the draft in
one multi-token step and returns its greedy token at every position. The committed
tokens are the longest prefix of the draft the target agrees with, plus one bonus
token (the target's token at the first disagreement, or after the full draft).
Like the reference, this is the acceptance core only; drafting is not wired into the
engine.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass
class SpeculativeConfig:
    draft_tokens: int = 4
    enabled: bool = False


@dataclass
class SpecAccept:
    accepted: int            # draft tokens accepted
    bonus: int               # the target's token after the accepted prefix

    def committed(self, draft: list[int]) -> list[int]:
        return list(draft[:self.accepted]) + [self.bonus]


def greedy_accept(draft: list[int], target: list[int]) -> SpecAccept:
    """target[i] is the target's greedy token after the context + draft[:i]
    (len(target) == len(draft) + 1)."""
    if len(target) != len(draft) + 1:
        raise ValueError("target must score every draft position plus one")
    n = 0
    while n < len(draft) and draft[n] == target[n]:
        n += 1
    return SpecAccept(n, target[n])
