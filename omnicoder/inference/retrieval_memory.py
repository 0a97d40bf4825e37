"""Retrieval memories for generation (reference src/omnicoder/inference/
retrieval_faiss.py, retrieval_memory.py, semantic_memory.py, retrieval_tokens.py).

ExternalRetrievalMemory: text chunks with L2-normalised embeddings (a hashing
bag-of-words embedder by default, or any callable), top-k cosine search with
numpy (FAISS is used when importable).  SemanticMemory: key -> fact store with
exponential relevance decay and reinforcement on access.  retrieval_prefix:
the token ids of the retrieved chunks to prepend to a prompt.
"""
from __future__ import annotations

import hashlib
import math
import re

import numpy as np


def hashing_embed(text: str, dim: int = 512) -> np.ndarray:
    v = np.zeros(dim, dtype=np.float32)
    for w in re.findall(r"\w+", text.lower()):
        h = int(hashlib.md5(w.encode()).hexdigest()[:8], 16)
        v[h % dim] += 1.0 if (h >> 31) & 1 else -1.0
    n = np.linalg.norm(v)
    return v / n if n > 0 else v


class ExternalRetrievalMemory:
    def __init__(self, embed=None, dim: int = 512):
        self.embed = embed or (lambda t: hashing_embed(t, dim))
        self.texts: list[str] = []
        self.vecs = np.zeros((0, dim), dtype=np.float32)
        try:
            import faiss  # noqa: F401
            self._faiss = True
        except ImportError:
            self._faiss = False

    def add(self, texts: list[str]) -> None:
        vs = np.stack([self.embed(t) for t in texts]).astype(np.float32)
        self.texts += list(texts)
        self.vecs = np.concatenate([self.vecs, vs]) if len(self.vecs) else vs

    def search(self, query: str, k: int = 3) -> list[tuple[str, float]]:
        if not self.texts:
            return []
        q = self.embed(query).astype(np.float32)
        s = self.vecs @ q
        idx = np.argsort(-s)[:k]
        return [(self.texts[i], float(s[i])) for i in idx]


class SemanticMemory:
    def __init__(self, half_life: float = 100.0):
        self.facts: dict = {}
        self.t = 0
        self.lam = math.log(2) / half_life

    def put(self, key: str, value, strength: float = 1.0) -> None:
        self.t += 1
        self.facts[key] = [value, strength, self.t]

    def relevance(self, key: str) -> float:
        v, s, t0 = self.facts[key]
        return s * math.exp(-self.lam * (self.t - t0))

    def get(self, key: str, reinforce: float = 0.5):
        self.t += 1
        if key not in self.facts:
            return None
        f = self.facts[key]
        f[1] = self.relevance(key) + reinforce
        f[2] = self.t
        return f[0]

    def top(self, n: int = 5) -> list:
        return sorted(self.facts, key=self.relevance, reverse=True)[:n]

    def forget(self, threshold: float = 0.05) -> int:
        drop = [k for k in self.facts if self.relevance(k) < threshold]
        for k in drop:
            del self.facts[k]
        return len(drop)


def retrieval_prefix(memory: ExternalRetrievalMemory, query: str, tokenize, k: int = 2, sep: list[int] | None = None):
    ids: list[int] = []
    for text, _ in memory.search(query, k):
        ids += tokenize(text) + (sep or [])
    return ids
