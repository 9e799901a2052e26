"""Exact-token-prefix snapshot cache (LRU over bytes and entry count).

Behaviour (harness/prefix_cache.rs:1-160): entries are keyed by an exact token
prefix; `longest_match` returns the longest cached key that is a STRICT prefix of
the query (at least one token must remain to prefill); inserting a key drops cached
entries that are strict prefixes of it (they are subsumed); eviction is LRU until
both the byte budget and the entry cap hold. Snapshots are opaque to the cache
(K/V + GDN conv and recurrent state, owned by the model's state pool).
"""
from __future__ import annotations

import threading
from collections import OrderedDict
from dataclasses import dataclass
from typing import Any, Callable


@dataclass
class PrefixEntry:
    tokens: tuple[int, ...]
    snapshot: Any
    nbytes: int


class PrefixCache:
    def __init__(self, budget_bytes: int = 1024 << 20, max_entries: int = 8,
                 on_evict: Callable[[Any], None] | None = None):
        self.budget = budget_bytes
        self.max_entries = max_entries
        self.on_evict = on_evict
        self._lru: "OrderedDict[tuple[int, ...], PrefixEntry]" = OrderedDict()
        self._bytes = 0
        self._lock = threading.Lock()
        self.hits = 0
        self.misses = 0

    def __len__(self) -> int:
        return len(self._lru)

    @property
    def nbytes(self) -> int:
        return self._bytes

    def longest_match(self, tokens: list[int] | tuple[int, ...]) -> PrefixEntry | None:
        q = tuple(tokens)
        with self._lock:
            best = None
            for key, ent in self._lru.items():
                n = len(key)
                if n < len(q) and q[:n] == key and (best is None or n > len(best.tokens)):
                    best = ent
            if best is not None:
                self._lru.move_to_end(best.tokens)
                self.hits += 1
            else:
                self.misses += 1
            return best

    def insert(self, tokens: list[int] | tuple[int, ...], snapshot: Any, nbytes: int) -> bool:
        key = tuple(tokens)
        if nbytes > self.budget:
            if self.on_evict:
                self.on_evict(snapshot)
            return False
        with self._lock:
            dropped = []
            for k in list(self._lru):
                if len(k) < len(key) and key[:len(k)] == k or k == key:
                    dropped.append(self._lru.pop(k))
            for d in dropped:
                self._bytes -= d.nbytes
            self._lru[key] = PrefixEntry(key, snapshot, nbytes)
            self._bytes += nbytes
            evicted = []
            while self._lru and (self._bytes > self.budget or len(self._lru) > self.max_entries):
                _, e = self._lru.popitem(last=False)
                self._bytes -= e.nbytes
                evicted.append(e)
        if self.on_evict:
            for e in dropped + evicted:
                if e.tokens != key or e.snapshot is not snapshot:
                    self.on_evict(e.snapshot)
        return True

    def remove_covering(self, tokens: list[int] | tuple[int, ...]) -> int:
        """Drop every entry whose key is a prefix of `tokens` (e.g. after a failed restore)."""
        q = tuple(tokens)
        with self._lock:
            gone = [k for k in self._lru if len(k) <= len(q) and q[:len(k)] == k]
            ents = [self._lru.pop(k) for k in gone]
            for e in ents:
                self._bytes -= e.nbytes
        if self.on_evict:
            for e in ents:
                self.on_evict(e.snapshot)
        return len(ents)

    def clear(self):
        with self._lock:
            ents = list(self._lru.values())
            self._lru.clear()
            self._bytes = 0
        if self.on_evict:
            for e in ents:
                self.on_evict(e.snapshot)


def stable_snapshot_cut(tokens: list[int], im_start_id: int | None) -> int:
    """Where to snapshot a chat prompt: one past the last `<|im_start|>` (the start of
    the assistant turn), so the next turn of the same conversation reuses everything
    before it (harness/candle.rs:6999). Without the marker: the whole prompt minus one."""
    if im_start_id is not None:
        for i in range(len(tokens) - 1, -1, -1):
            if tokens[i] == im_start_id:
                return i + 1 if i + 1 < len(tokens) else i
    return max(0, len(tokens) - 1)
