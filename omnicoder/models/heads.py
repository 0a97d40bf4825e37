"""Output-head utilities.

FastHeadShortlist (reference src/omnicoder/modeling/utils/fast_head.py:9-220):
exact argmax over a large vocabulary from a low-dimensional shortlist.  A
strided subset S of the hidden dims gives coarse scores h_S . W_S; by
Cauchy-Schwarz the rest of each score is bounded by |h_R| * |W_R[v]|.  The
top-k candidates by coarse score are rescored exactly; the argmax is exact once
the best exact score beats every unscored candidate's upper bound, otherwise
the shortlist is widened (x2) and the check repeats.

ContinuousLatentHead / ConceptLatentHead: projections of the hidden state to
small continuous latents (reference multimodal/aligner.py:54-97).
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F


class FastHeadShortlist:
    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None = None, sub_dims: int = 128):
        W = weight.detach().float()
        V, D = W.shape
        k = max(8, min(D, sub_dims))
        stride = max(1, D // k)
        sub = torch.arange(0, D, stride, device=W.device)[:k]
        mask = torch.ones(D, dtype=torch.bool, device=W.device)
        mask[sub] = False
        self.sub, self.res = sub, mask.nonzero().squeeze(1)
        self.W, self.b = W, (None if bias is None else bias.detach().float())
        self.W_sub_t = W[:, sub].t().contiguous()
        self.res_norm = W[:, self.res].norm(dim=1) if self.res.numel() else torch.zeros(V, device=W.device)

    @classmethod
    def from_linear(cls, lm_head: nn.Linear, sub_dims: int = 128) -> "FastHeadShortlist":
        return cls(lm_head.weight, lm_head.bias, sub_dims)

    @torch.no_grad()
    def argmax(self, hidden: torch.Tensor, initial_k: int = 2048, widen_factor: float = 2.0) -> torch.Tensor:
        """hidden [B, C] or [B, T, C] (last position) -> next ids [B, 1], exact."""
        h = (hidden[:, -1] if hidden.dim() == 3 else hidden).float()
        coarse = h[:, self.sub] @ self.W_sub_t
        if self.b is not None:
            coarse = coarse + self.b
        bound = h[:, self.res].norm(dim=1, keepdim=True) * self.res_norm[None]   # |residual score| bound
        V = coarse.shape[1]
        out = torch.empty(h.shape[0], 1, dtype=torch.long, device=h.device)
        for i in range(h.shape[0]):
            k = min(V, initial_k)
            upper = coarse[i] + bound[i]
            while True:
                cand = torch.topk(upper, k).indices
                exact = self.W[cand] @ h[i] + (0 if self.b is None else self.b[cand])
                best = int(exact.argmax())
                if k >= V:
                    out[i, 0] = cand[best]
                    break
                rest = torch.ones(V, dtype=torch.bool, device=h.device)
                rest[cand] = False
                if exact[best] >= upper[rest].max():
                    out[i, 0] = cand[best]
                    break
                k = min(V, int(k * widen_factor))
        return out


class ContinuousLatentHead(nn.Module):
    def __init__(self, d_model: int, latent_dim: int = 16):
        super().__init__()
        self.proj = nn.Sequential(nn.LayerNorm(d_model), nn.Linear(d_model, d_model), nn.GELU(),
                                  nn.Linear(d_model, latent_dim))

    def forward(self, h):
        return self.proj(h)


class ConceptLatentHead(nn.Module):
    """Last-position projection to a unit-norm concept embedding."""

    def __init__(self, d_model: int, embed_dim: int = 256):
        super().__init__()
        self.net = nn.Sequential(nn.LayerNorm(d_model), nn.Linear(d_model, d_model), nn.GELU(),
                                 nn.Linear(d_model, embed_dim))

    def forward(self, h):
        return F.normalize(self.net(h[:, -1] if h.dim() == 3 else h), dim=-1)
