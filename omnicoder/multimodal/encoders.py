"""Small modality encoders (reference modeling/multimodal/vision_encoder.py,
vqvae.py, audio_tokenizer.py, fusion.py MelProjector).

PatchEncoder: ViT-style image encoder (conv patchify + learned positions +
pre-norm transformer layers) -> [B, patches, dim].
VectorQuantizer: nearest-codebook quantisation with the straight-through
estimator and the VQ-VAE codebook/commitment loss; `encode` returns codes.
MelFrontend: log-mel spectrogram (torch.stft with a triangular mel filterbank)
followed by a linear projection.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F


class PatchEncoder(nn.Module):
    def __init__(self, image_size: int = 224, patch: int = 16, dim: int = 192, depth: int = 4, heads: int = 3,
                 in_ch: int = 3):
        super().__init__()
        self.proj = nn.Conv2d(in_ch, dim, patch, patch)
        n = (image_size // patch) ** 2
        self.pos = nn.Parameter(torch.randn(1, n + 1, dim) * 0.02)
        self.cls = nn.Parameter(torch.zeros(1, 1, dim))
        layer = nn.TransformerEncoderLayer(dim, heads, 4 * dim, dropout=0.0, batch_first=True, norm_first=True,
                                           activation="gelu")
        self.blocks = nn.TransformerEncoder(layer, depth, enable_nested_tensor=False)
        self.norm = nn.LayerNorm(dim)

    def forward(self, img):
        x = self.proj(img).flatten(2).transpose(1, 2)
        x = torch.cat([self.cls.expand(x.shape[0], -1, -1), x], 1) + self.pos[:, :x.shape[1] + 1]
        return self.norm(self.blocks(x))


class VectorQuantizer(nn.Module):
    def __init__(self, codebook_size: int = 8192, dim: int = 64, beta: float = 0.25):
        super().__init__()
        self.codebook = nn.Embedding(codebook_size, dim)
        nn.init.uniform_(self.codebook.weight, -1.0 / codebook_size, 1.0 / codebook_size)
        self.beta = beta

    def encode(self, z):
        flat = z.reshape(-1, z.shape[-1])
        d = (flat.pow(2).sum(1, keepdim=True) - 2 * flat @ self.codebook.weight.t()
             + self.codebook.weight.pow(2).sum(1)[None])
        return d.argmin(1).view(z.shape[:-1])

    def forward(self, z):
        codes = self.encode(z)
        q = self.codebook(codes)
        loss = F.mse_loss(q, z.detach()) + self.beta * F.mse_loss(z, q.detach())
        return z + (q - z).detach(), codes, loss


def mel_filterbank(n_mels: int, n_fft: int, sr: int) -> torch.Tensor:
    def hz2mel(f):
        return 2595.0 * math.log10(1.0 + f / 700.0)

    def mel2hz(m):
        return 700.0 * (10 ** (m / 2595.0) - 1.0)
    mels = torch.linspace(hz2mel(0.0), hz2mel(sr / 2), n_mels + 2)
    hz = torch.tensor([mel2hz(float(m)) for m in mels])
    bins = torch.floor((n_fft + 1) * hz / sr).long()
    fb = torch.zeros(n_mels, n_fft // 2 + 1)
    for i in range(n_mels):
        a, b, c = int(bins[i]), int(bins[i + 1]), int(bins[i + 2])
        for k in range(a, b):
            fb[i, k] = (k - a) / max(1, b - a)
        for k in range(b, c):
            fb[i, k] = (c - k) / max(1, c - b)
    return fb


class MelFrontend(nn.Module):
    def __init__(self, n_mels: int = 80, out_dim: int = 384, sr: int = 16000, n_fft: int = 400, hop: int = 160):
        super().__init__()
        self.n_fft, self.hop = n_fft, hop
        self.register_buffer("fb", mel_filterbank(n_mels, n_fft, sr), persistent=False)
        self.register_buffer("win", torch.hann_window(n_fft), persistent=False)
        self.proj = nn.Linear(n_mels, out_dim)

    def mel(self, wav):
        spec = torch.stft(wav, self.n_fft, self.hop, window=self.win, return_complex=True).abs().pow(2)
        return torch.log(self.fb @ spec + 1e-6).transpose(1, 2)      # [B, frames, n_mels]

    def forward(self, wav):
        return self.proj(self.mel(wav))
