"""Cross-modal alignment (reference src/omnicoder/modeling/multimodal/aligner.py:1-194,
fusion.py grounding / segmentation heads, av-sync utilities).

PreAligner: per-modality projections into one shared embedding space (mean
pooled, L2-normalised).  CrossModalVerifier: a mini-CLIP scorer (learned
temperature, cosine similarity) with the symmetric InfoNCE loss `clip_loss`.
GroundingHead: box regression [cx, cy, w, h] in [0, 1] from (text, image
patch) features by attention pooling.  SegmentationHead: per-patch mask
logits upsampled to the image size.  av_offset: audio/video lag (in frames)
that maximises the cross-correlation of per-frame embeddings.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F


class PreAligner(nn.Module):
    def __init__(self, dims: dict, shared: int = 256):
        super().__init__()
        self.proj = nn.ModuleDict({k: nn.Linear(d, shared) for k, d in dims.items()})

    def forward(self, modality: str, feats: torch.Tensor) -> torch.Tensor:
        x = feats.mean(1) if feats.dim() == 3 else feats
        return F.normalize(self.proj[modality](x), dim=-1)


def clip_loss(a: torch.Tensor, b: torch.Tensor, logit_scale: torch.Tensor) -> torch.Tensor:
    logits = logit_scale.exp() * a @ b.t()
    target = torch.arange(a.shape[0], device=a.device)
    return 0.5 * (F.cross_entropy(logits, target) + F.cross_entropy(logits.t(), target))


class CrossModalVerifier(nn.Module):
    def __init__(self, dims: dict, shared: int = 256):
        super().__init__()
        self.align = PreAligner(dims, shared)
        self.logit_scale = nn.Parameter(torch.tensor(math.log(1 / 0.07)))

    def score(self, ma: str, a: torch.Tensor, mb: str, b: torch.Tensor) -> torch.Tensor:
        return (self.align(ma, a) * self.align(mb, b)).sum(-1)

    def loss(self, ma: str, a: torch.Tensor, mb: str, b: torch.Tensor) -> torch.Tensor:
        return clip_loss(self.align(ma, a), self.align(mb, b), self.logit_scale)


class GroundingHead(nn.Module):
    def __init__(self, dim: int, heads: int = 4):
        super().__init__()
        self.attn = nn.MultiheadAttention(dim, heads, batch_first=True)
        self.box = nn.Sequential(nn.Linear(dim, dim), nn.GELU(), nn.Linear(dim, 4))

    def forward(self, text_feat: torch.Tensor, patches: torch.Tensor) -> torch.Tensor:
        q = text_feat.mean(1, keepdim=True)
        pooled, _ = self.attn(q, patches, patches)
        return torch.sigmoid(self.box(pooled.squeeze(1)))


class SegmentationHead(nn.Module):
    def __init__(self, dim: int, n_classes: int = 1):
        super().__init__()
        self.cls = nn.Linear(dim, n_classes)

    def forward(self, patches: torch.Tensor, grid: int, image_size: int) -> torch.Tensor:
        B, N, _ = patches.shape
        logits = self.cls(patches[:, -grid * grid:]).transpose(1, 2).reshape(B, -1, grid, grid)
        return F.interpolate(logits, size=(image_size, image_size), mode="bilinear", align_corners=False)


def av_offset(audio_emb: torch.Tensor, video_emb: torch.Tensor, max_lag: int = 10) -> int:
    """Lag L (audio frame t matches video frame t + L) with the highest mean cosine similarity."""
    a = F.normalize(audio_emb, dim=-1)
    v = F.normalize(video_emb, dim=-1)
    best, best_l = -2.0, 0
    T = min(a.shape[0], v.shape[0])
    for lag in range(-max_lag, max_lag + 1):
        lo, hi = max(0, -lag), min(T, T - lag)
        if hi - lo <= 0:
            continue
        s = (a[lo:hi] * v[lo + lag:hi + lag]).sum(-1).mean().item()
        if s > best:
            best, best_l = s, lag
    return best_l
