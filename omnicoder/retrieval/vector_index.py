"""Dense vector search on the device, and a chunked-text retriever on top of it
(reference src/omnicoder/inference/retrieval_faiss.py:35-160, which hashes
TF-IDF vectors into a FAISS index; FAISS is not a dependency here).

VectorIndex       exact search: scores = Q X^T (inner product, or cosine on
                  normalised rows, or negative squared L2) as one GEMM per
                  database chunk, merged top-k across chunks, so the database
                  can exceed what one score matrix should hold.  On a CUDA device
                  the GEMM runs on the tensor cores.
IVFIndex          inverted lists: k-means coarse centroids (on the device), each
                  vector stored under its nearest centroid; a query scans the
                  `nprobe` closest lists only.
TextRetriever     overlapping word chunks of a corpus, hashed TF-IDF vectors
                  (signed feature hashing, log-scaled term frequency, IDF from
                  the corpus), cosine search; returns (score, text) chunks.
"""
from __future__ import annotations

import math
import re
from collections import Counter
from dataclasses import dataclass

import torch


def _scores(q: torch.Tensor, x: torch.Tensor, metric: str) -> torch.Tensor:
    if metric in ("ip", "cosine"):
        return q @ x.t()
    if metric == "l2":
        return 2 * (q @ x.t()) - (x * x).sum(1)[None] - (q * q).sum(1)[:, None]
    raise ValueError(f"unknown metric {metric!r}")


class VectorIndex:
    def __init__(self, dim: int, metric: str = "cosine", device=None, dtype=torch.float32, chunk: int = 65536):
        self.dim, self.metric, self.chunk = dim, metric, chunk
        self.device = torch.device(device or "cpu")
        self.dtype = dtype
        self.x = torch.empty(0, dim, device=self.device, dtype=dtype)

    def _prep(self, v: torch.Tensor) -> torch.Tensor:
        v = v.to(self.device, self.dtype).reshape(-1, self.dim)
        return torch.nn.functional.normalize(v, dim=1) if self.metric == "cosine" else v

    def add(self, vectors: torch.Tensor) -> None:
        self.x = torch.cat([self.x, self._prep(vectors)], 0)

    def __len__(self) -> int:
        return self.x.shape[0]

    @torch.no_grad()
    def search(self, queries: torch.Tensor, k: int = 5):
        """-> (scores [Q, k] higher is better (negative squared distance for l2), ids [Q, k])."""
        q = self._prep(queries)
        k = min(k, len(self))
        best_s = torch.full((q.shape[0], 0), float("-inf"), device=self.device)
        best_i = torch.empty(q.shape[0], 0, dtype=torch.long, device=self.device)
        for s in range(0, len(self), self.chunk):
            sc = _scores(q, self.x[s:s + self.chunk], self.metric).float()
            v, i = sc.topk(min(k, sc.shape[1]), dim=1)
            best_s, order = torch.cat([best_s, v], 1).topk(min(k, best_s.shape[1] + v.shape[1]), dim=1)
            best_i = torch.cat([best_i, i + s], 1).gather(1, order)
        return best_s, best_i


class IVFIndex:
    def __init__(self, dim: int, n_lists: int = 64, metric: str = "cosine", nprobe: int = 8, device=None, seed: int = 0):
        self.dim, self.n_lists, self.metric, self.nprobe, self.seed = dim, n_lists, metric, nprobe, seed
        self.device = torch.device(device or "cpu")
        self.centroids = None
        self.lists: list[VectorIndex] = []
        self.ids: list[torch.Tensor] = []
        self.count = 0

    def _prep(self, v):
        v = v.to(self.device, torch.float32).reshape(-1, self.dim)
        return torch.nn.functional.normalize(v, dim=1) if self.metric == "cosine" else v

    @torch.no_grad()
    def train(self, sample: torch.Tensor, iters: int = 20) -> None:
        x = self._prep(sample)
        g = torch.Generator(device="cpu").manual_seed(self.seed)
        c = x[torch.randperm(x.shape[0], generator=g)[:self.n_lists].to(x.device)].clone()
        for _ in range(iters):
            a = _scores(x, c, "l2").argmax(1)
            for j in range(c.shape[0]):
                m = a == j
                if m.any():
                    c[j] = x[m].mean(0)
        self.centroids = c
        self.lists = [VectorIndex(self.dim, self.metric, self.device) for _ in range(c.shape[0])]
        self.ids = [torch.empty(0, dtype=torch.long, device=self.device) for _ in range(c.shape[0])]

    @torch.no_grad()
    def add(self, vectors: torch.Tensor) -> None:
        if self.centroids is None:
            self.train(vectors)
        x = self._prep(vectors)
        a = _scores(x, self.centroids, "l2").argmax(1)
        ids = torch.arange(self.count, self.count + x.shape[0], device=self.device)
        for j in range(self.centroids.shape[0]):
            m = a == j
            if m.any():
                self.lists[j].add(x[m])
                self.ids[j] = torch.cat([self.ids[j], ids[m]])
        self.count += x.shape[0]

    @torch.no_grad()
    def search(self, queries: torch.Tensor, k: int = 5):
        q = self._prep(queries)
        probe = _scores(q, self.centroids, "l2").topk(min(self.nprobe, self.centroids.shape[0]), dim=1).indices
        out_s = torch.full((q.shape[0], k), float("-inf"), device=self.device)
        out_i = torch.full((q.shape[0], k), -1, dtype=torch.long, device=self.device)
        for r in range(q.shape[0]):
            ss, ii = [], []
            for j in probe[r].tolist():
                if len(self.lists[j]):
                    s, i = self.lists[j].search(q[r:r + 1], k)
                    ss.append(s[0])
                    ii.append(self.ids[j][i[0]])
            if ss:
                s, i = torch.cat(ss), torch.cat(ii)
                top = s.topk(min(k, s.numel()))
                out_s[r, :top.values.numel()] = top.values
                out_i[r, :top.values.numel()] = i[top.indices]
        return out_s, out_i


_WORD = re.compile(r"[A-Za-z0-9_]+")


@dataclass
class RetrievedChunk:
    score: float
    text: str
    index: int


class TextRetriever:
    def __init__(self, texts: list[str], dim: int = 4096, chunk_words: int = 128, stride: int = 96, device=None):
        self.dim = dim
        self.chunks: list[str] = []
        for t in texts:
            words = t.split()
            for s in range(0, max(1, len(words) - chunk_words + stride), stride):
                piece = " ".join(words[s:s + chunk_words])
                if piece:
                    self.chunks.append(piece)
        toks = [self._tokens(c) for c in self.chunks]
        df = Counter(w for ts in toks for w in set(ts))
        n = max(1, len(toks))
        self.idf = {w: math.log((1 + n) / (1 + d)) + 1.0 for w, d in df.items()}
        self.index = VectorIndex(dim, "cosine", device)
        if toks:
            self.index.add(torch.stack([self._vec(ts) for ts in toks]))

    @staticmethod
    def _tokens(text: str) -> list[str]:
        return [w.lower() for w in _WORD.findall(text)]

    def _vec(self, toks: list[str]) -> torch.Tensor:
        v = torch.zeros(self.dim)
        for w, c in Counter(toks).items():
            h = hash_token(w)
            v[h % self.dim] += (1.0 if (h >> 20) & 1 else -1.0) * (1.0 + math.log(c)) * self.idf.get(w, 1.0)
        return v

    def search(self, query: str, k: int = 3) -> list[RetrievedChunk]:
        if not self.chunks:
            return []
        s, i = self.index.search(self._vec(self._tokens(query))[None], k)
        return [RetrievedChunk(float(a), self.chunks[int(b)], int(b)) for a, b in zip(s[0], i[0])]


def hash_token(w: str) -> int:
    """Stable 32-bit FNV-1a hash (Python's str hash is salted per process)."""
    h = 2166136261
    for byte in w.encode():
        h = ((h ^ byte) * 16777619) & 0xFFFFFFFF
    return h
