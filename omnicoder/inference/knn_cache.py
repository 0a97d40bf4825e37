"""kNN-LM cache (reference src/omnicoder/inference/knn_cache.py:18-287).

Stores (hidden state, next token) pairs; at decode time the k nearest stored
states (L2) vote for their next tokens with weights softmax(-d / temperature),
and the resulting distribution is mixed into the model's:
p = (1 - lam) * p_model + lam * p_knn.  Keys live on the device of the
first `add`; search is one matmul against all keys (exact), chunked."""
from __future__ import annotations

import torch


class KNNCache:
    def __init__(self, dim: int, capacity: int = 100_000, k: int = 8, temperature: float = 1.0, lam: float = 0.25):
        self.dim, self.capacity, self.k, self.temperature, self.lam = dim, capacity, k, temperature, lam
        self.keys: torch.Tensor | None = None
        self.vals: torch.Tensor | None = None

    def __len__(self):
        return 0 if self.keys is None else self.keys.shape[0]

    @torch.no_grad()
    def add(self, hidden: torch.Tensor, next_ids: torch.Tensor) -> None:
        h = hidden.reshape(-1, self.dim).float()
        v = next_ids.reshape(-1).long().to(h.device)
        self.keys = h if self.keys is None else torch.cat([self.keys, h])[-self.capacity:]
        self.vals = v if self.vals is None else torch.cat([self.vals, v])[-self.capacity:]

    @torch.no_grad()
    def query(self, hidden: torch.Tensor, vocab: int) -> torch.Tensor:
        """hidden [B, D] -> kNN distribution [B, V]."""
        q = hidden.reshape(-1, self.dim).float()
        out = torch.zeros(q.shape[0], vocab, device=q.device)
        if not len(self):
            return out
        d = (q * q).sum(1, keepdim=True) - 2 * q @ self.keys.t() + (self.keys * self.keys).sum(1)[None]
        k = min(self.k, self.keys.shape[0])
        dist, idx = torch.topk(d, k, dim=1, largest=False)
        w = torch.softmax(-dist / self.temperature, dim=1)
        return out.scatter_add_(1, self.vals[idx], w)

    @torch.no_grad()
    def blend(self, logits: torch.Tensor, hidden: torch.Tensor) -> torch.Tensor:
        """Mix into log-probabilities: log((1 - lam) softmax(logits) + lam p_knn)."""
        p = torch.softmax(logits.float(), -1)
        if len(self):
            p = (1 - self.lam) * p + self.lam * self.query(hidden, logits.shape[-1])
        return torch.log(p.clamp_min(1e-30))

    def save(self, path: str) -> None:
        torch.save({"keys": self.keys, "vals": self.vals, "cfg": (self.dim, self.capacity, self.k, self.temperature,
                                                                 self.lam)}, path)

    @classmethod
    def load(cls, path: str) -> "KNNCache":
        d = torch.load(path, weights_only=False)
        c = cls(*d["cfg"])
        c.keys, c.vals = d["keys"], d["vals"]
        return c
