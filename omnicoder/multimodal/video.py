"""Video and 3D latent modules (reference src/omnicoder/modeling/multimodal/video_encoder.py,
latent3d.py, latent_refiner.py, video_interpolate.py).

TemporalMixer        gated (GELU-GLU) projection + depthwise 1-D convolution over time, [B, T, C] -> [B, T, C]
VideoEncoder         per-frame ViT (PatchEncoder) CLS features mixed over time -> ([B, T, C], pooled [B, C])
VoxelLatentHead      the last hidden token -> a [B, D, H, W] voxel density grid
OrthoRenderer        voxel densities -> RGB by per-slice colours and front-to-back alpha compositing
LatentRefiner        residual, gated MLP refinement of continuous latents ([B, D] or [B, T, D]),
                     optionally followed by a depthwise temporal convolution
LatentInterpolator   latents between two keyframes at evenly spaced times, predicted from (z0, z1, tau)
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .encoders import PatchEncoder


class TemporalMixer(nn.Module):
    """causal=True pads only the past side, so the output at frame t sees frames <= t."""

    def __init__(self, d_model: int, kernel_size: int = 5, expansion: int = 2, causal: bool = False):
        super().__init__()
        hidden = d_model * expansion
        self.inp = nn.Linear(d_model, 2 * hidden, bias=False)
        self.conv = nn.Conv1d(hidden, hidden, kernel_size, groups=hidden)
        self.out = nn.Linear(hidden, d_model, bias=False)
        k = kernel_size
        self.pad = (k - 1, 0) if causal else (k // 2, k - 1 - k // 2)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        a, b = self.inp(x).chunk(2, dim=-1)
        y = self.conv(F.pad((a * F.gelu(b)).transpose(1, 2), self.pad)).transpose(1, 2)
        return self.out(y)


class VideoEncoder(nn.Module):
    """frames [B, T, 3, S, S] -> (per-frame features [B, T, dim], pooled [B, dim])."""

    def __init__(self, image_size: int = 224, patch: int = 16, dim: int = 192, depth: int = 4, heads: int = 3,
                 temporal_kernel: int = 5):
        super().__init__()
        self.frames = PatchEncoder(image_size, patch, dim, depth, heads)
        self.temporal = TemporalMixer(dim, temporal_kernel)
        self.norm = nn.LayerNorm(dim)

    def forward(self, video: torch.Tensor):
        B, T = video.shape[:2]
        cls = self.frames(video.flatten(0, 1))[:, 0].view(B, T, -1)
        feats = self.norm(cls + self.temporal(cls))
        return feats, feats.mean(1)


class VoxelLatentHead(nn.Module):
    def __init__(self, d_model: int, depth: int = 16, height: int = 32, width: int = 32, hidden: int = 256):
        super().__init__()
        self.shape = (depth, height, width)
        self.net = nn.Sequential(nn.LayerNorm(d_model), nn.Linear(d_model, hidden), nn.GELU(),
                                 nn.Linear(hidden, depth * height * width))

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        code = hidden[:, -1]
        return self.net(code).view(code.shape[0], *self.shape)


class OrthoRenderer(nn.Module):
    """vox [B, D, H, W] (any range) -> image [B, 3, out_h, out_w]; slice 0 is nearest the camera."""

    def __init__(self, depth: int = 16, out_h: int = 256, out_w: int = 256):
        super().__init__()
        self.size = (depth, out_h, out_w)
        self.color = nn.Parameter(torch.randn(depth, 3) * 0.1)

    def forward(self, vox: torch.Tensor) -> torch.Tensor:
        x = F.interpolate(vox.unsqueeze(1), size=self.size, mode="trilinear", align_corners=False).squeeze(1)
        alpha = torch.sigmoid(x)                                            # [B, D, H, W]
        trans = torch.cumprod(torch.cat([torch.ones_like(alpha[:, :1]), 1 - alpha[:, :-1]], 1), 1)
        weight = trans * alpha                                              # front-to-back compositing
        return torch.einsum("bdhw,dc->bchw", weight, torch.sigmoid(self.color))


class LatentRefiner(nn.Module):
    def __init__(self, latent_dim: int, hidden_mult: int = 2, temporal: bool = False, kernel_size: int = 3):
        super().__init__()
        hidden = max(1, hidden_mult) * latent_dim
        self.norm = nn.LayerNorm(latent_dim)
        self.up = nn.Linear(latent_dim, hidden, bias=False)
        self.down = nn.Linear(hidden, latent_dim, bias=False)
        self.gate = nn.Parameter(torch.tensor(1.0))
        self.tconv = (nn.Conv1d(latent_dim, latent_dim, kernel_size, padding=kernel_size // 2, groups=latent_dim)
                      if temporal else None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() not in (2, 3):
            raise ValueError("LatentRefiner expects [B, D] or [B, T, D]")
        y = x + self.gate * self.down(F.gelu(self.up(self.norm(x))))
        if x.dim() == 3 and self.tconv is not None:
            y = self.tconv(y.transpose(1, 2)).transpose(1, 2)
        return y


class LatentInterpolator(nn.Module):
    """z0, z1 [B, T, D] -> [B, steps, T, D] at tau = 0 .. 1."""

    def __init__(self, latent_dim: int = 16, hidden: int = 64):
        super().__init__()
        self.net = nn.Sequential(nn.Linear(2 * latent_dim + 1, hidden), nn.GELU(), nn.Linear(hidden, latent_dim))

    def forward(self, z0: torch.Tensor, z1: torch.Tensor, steps: int) -> torch.Tensor:
        B, T, D = z0.shape
        tau = torch.linspace(0, 1, steps, device=z0.device, dtype=z0.dtype).view(1, steps, 1, 1).expand(B, steps, T, 1)
        a = z0.unsqueeze(1).expand(B, steps, T, D)
        b = z1.unsqueeze(1).expand(B, steps, T, D)
        return self.net(torch.cat([a, b, tau], -1))
