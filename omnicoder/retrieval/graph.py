"""Graph retrieval and logit biasing (reference src/omnicoder/retrieval/graphrag.py:1-304,
sfb/fusion/cross_bias.py:1-168).

GraphRAG: entities (capitalised words, identifiers, numbers) are nodes; two
entities are linked when they occur in the same passage.  A query's entities
seed a personalised-PageRank-style walk (restart probability `alpha`) over the
graph; passages are ranked by the mass on their entities.  `logit_bias_from_text`
turns retrieved text into an additive bias over the token ids that text
contains (a vector to add to the next-token logits).
"""
from __future__ import annotations

import collections
import re

import torch

_ENT = re.compile(r"\b([A-Z][A-Za-z0-9_]+|[a-z_]+\(\)|\d+(?:\.\d+)?)\b")


def entities(text: str) -> set[str]:
    return set(m.group(1).lower() for m in _ENT.finditer(text))


class GraphRAG:
    def __init__(self, alpha: float = 0.15, iters: int = 20):
        self.alpha, self.iters = alpha, iters
        self.passages: list[str] = []
        self.ents: list[set[str]] = []
        self.adj: dict[str, collections.Counter] = collections.defaultdict(collections.Counter)

    def add(self, passages: list[str]) -> "GraphRAG":
        for p in passages:
            e = entities(p)
            self.passages.append(p)
            self.ents.append(e)
            for a in e:
                for b in e:
                    if a != b:
                        self.adj[a][b] += 1
        return self

    def scores(self, query: str) -> dict[str, float]:
        seeds = [e for e in entities(query) if e in self.adj]
        if not seeds:
            return {}
        r0 = {e: 1.0 / len(seeds) for e in seeds}
        r = dict(r0)
        for _ in range(self.iters):
            nxt = collections.defaultdict(float)
            for a, m in r.items():
                tot = sum(self.adj[a].values()) or 1
                for b, w in self.adj[a].items():
                    nxt[b] += (1 - self.alpha) * m * w / tot
            for e, m in r0.items():
                nxt[e] += self.alpha * m
            r = nxt
        return dict(r)

    def retrieve(self, query: str, k: int = 3) -> list[tuple[float, str]]:
        s = self.scores(query)
        ranked = sorted(((sum(s.get(e, 0.0) for e in ents), p) for ents, p in zip(self.ents, self.passages)),
                        key=lambda t: -t[0])
        return [t for t in ranked[:k] if t[0] > 0]


def logit_bias_from_text(text: str, tokenizer, vocab_size: int, strength: float = 1.0) -> torch.Tensor:
    bias = torch.zeros(vocab_size)
    ids = [i for i in tokenizer.encode(text) if 0 <= i < vocab_size]
    if ids:
        bias[torch.tensor(ids)] = strength
    return bias
