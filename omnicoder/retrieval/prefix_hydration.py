"""Prefix hydration: reuse the decode state of an earlier, similar prompt (reference
src/omnicoder/retrieval/prefix_hydration.py:1-26, which only defines the fingerprint).

``semantic_fingerprint`` hashes each lower-cased word with SHA-1 into one of ``num_buckets`` counters, so the
fingerprints of a session store written by either implementation compare equal. ``PrefixHydrationStore`` keeps
up to ``capacity`` saved states (a KV cache, landmarks, memory rows: whatever the caller saves) keyed by their
prompt's fingerprint, least recently used first out. ``lookup`` returns the stored entry whose fingerprint has
the highest cosine similarity with the new prompt's, if it reaches ``threshold``. When both prompts come with
token ids, it also returns the length of their common token prefix: the number of cached positions that can be
kept (crop the cache to it, then prefill only the rest); an entry sharing no leading token is not a hit.
"""
from __future__ import annotations

import hashlib
import math
from collections import OrderedDict
from dataclasses import dataclass
from typing import Any, Sequence


def semantic_fingerprint(text: str, num_buckets: int = 256) -> list[int]:
    out = [0] * max(1, int(num_buckets))
    for w in text.lower().split():
        out[int(hashlib.sha1(w.encode("utf-8")).hexdigest(), 16) % len(out)] += 1
    return out


def _cosine(a: Sequence[int], b: Sequence[int]) -> float:
    na = math.sqrt(sum(x * x for x in a))
    nb = math.sqrt(sum(x * x for x in b))
    if na == 0.0 or nb == 0.0:
        return 0.0
    return sum(x * y for x, y in zip(a, b)) / (na * nb)


def common_prefix_len(a: Sequence[int], b: Sequence[int]) -> int:
    n = 0
    for x, y in zip(a, b):
        if x != y:
            break
        n += 1
    return n


@dataclass
class Hydration:
    state: Any
    similarity: float
    reuse_tokens: int | None  # common token prefix; None when either prompt came without token ids
    key: str


class PrefixHydrationStore:
    def __init__(self, capacity: int = 64, threshold: float = 0.9, num_buckets: int = 256):
        if capacity < 1 or not 0.0 <= threshold <= 1.0:
            raise ValueError("capacity must be >= 1 and threshold in [0, 1]")
        self.capacity, self.threshold, self.num_buckets = capacity, threshold, num_buckets
        self._entries: OrderedDict[str, tuple[list[int], list[int] | None, Any]] = OrderedDict()

    def __len__(self) -> int:
        return len(self._entries)

    def put(self, text: str, state: Any, token_ids: Sequence[int] | None = None) -> str:
        """Save ``state`` for the prompt ``text``; returns its key (the SHA-1 of the text)."""
        key = hashlib.sha1(text.encode("utf-8")).hexdigest()
        self._entries.pop(key, None)
        self._entries[key] = (semantic_fingerprint(text, self.num_buckets),
                              None if token_ids is None else [int(t) for t in token_ids], state)
        while len(self._entries) > self.capacity:
            self._entries.popitem(last=False)
        return key

    def lookup(self, text: str, token_ids: Sequence[int] | None = None) -> Hydration | None:
        fp = semantic_fingerprint(text, self.num_buckets)
        best: Hydration | None = None
        for key, (efp, eids, state) in self._entries.items():
            sim = _cosine(fp, efp)
            if sim < self.threshold or (best is not None and sim <= best.similarity):
                continue
            reuse = None if token_ids is None or eids is None else common_prefix_len(eids, token_ids)
            if reuse == 0:
                continue
            best = Hydration(state, sim, reuse, key)
        if best is not None:
            self._entries.move_to_end(best.key)
        return best

    def clear(self) -> None:
        self._entries.clear()
