"""Image / video / audio VQ-VAEs and decoders (reference
src/omnicoder/modeling/multimodal/vqvae.py:1-347, video_vq / audio VQ trainers,
vocoder in the audio pipeline).

ImageVQVAE: strided conv encoder (downsample 2^levels) -> VectorQuantizer ->
transposed-conv decoder; `encode` gives [B, h, w] codes for the unified
vocabulary, `decode` reconstructs images from codes.
VideoVQVAE: the image VQ-VAE per frame plus a temporal 1-D conv over the
latent grid (frames share the codebook); codes [B, T, h, w].
AudioVQ: mel front end -> conv encoder over time -> VectorQuantizer; codes
[B, frames'].
MelVocoder: transposed-conv upsampling stack (mel frames -> waveform, the
HiFi-GAN generator shape without its discriminators), for decoding audio codes.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .encoders import MelFrontend, VectorQuantizer


def _down(cin, cout):
    return nn.Sequential(nn.Conv2d(cin, cout, 4, 2, 1), nn.GroupNorm(8, cout), nn.SiLU())


def _up(cin, cout):
    return nn.Sequential(nn.ConvTranspose2d(cin, cout, 4, 2, 1), nn.GroupNorm(8, cout), nn.SiLU())


class ImageVQVAE(nn.Module):
    def __init__(self, in_ch: int = 3, width: int = 64, levels: int = 3, code_dim: int = 64,
                 codebook_size: int = 8192):
        super().__init__()
        enc, c = [], in_ch
        for i in range(levels):
            enc.append(_down(c, width * 2 ** i))
            c = width * 2 ** i
        self.enc = nn.Sequential(*enc, nn.Conv2d(c, code_dim, 1))
        self.vq = VectorQuantizer(codebook_size, code_dim)
        dec = [nn.Conv2d(code_dim, c, 1)]
        for i in reversed(range(levels)):
            cout = width * 2 ** (i - 1) if i > 0 else width
            dec.append(_up(c, cout))
            c = cout
        self.dec = nn.Sequential(*dec, nn.Conv2d(c, in_ch, 3, 1, 1))

    def _latent(self, img):
        return self.enc(img).permute(0, 2, 3, 1)                 # [B, h, w, D]

    def encode(self, img):
        return self.vq.encode(self._latent(img))

    def decode(self, codes):
        q = self.vq.codebook(codes).permute(0, 3, 1, 2)
        return self.dec(q)

    def forward(self, img):
        zq, codes, vq_loss = self.vq(self._latent(img))
        rec = self.dec(zq.permute(0, 3, 1, 2))
        return rec, codes, F.mse_loss(rec, img) + vq_loss


class VideoVQVAE(nn.Module):
    def __init__(self, **kw):
        super().__init__()
        self.image = ImageVQVAE(**kw)
        d = self.image.vq.codebook.weight.shape[1]
        self.temporal = nn.Conv1d(d, d, 3, padding=1)

    def _latent(self, video):                                    # video [B, T, C, H, W]
        B, T = video.shape[:2]
        z = self.image._latent(video.flatten(0, 1))               # [B*T, h, w, D]
        h, w, D = z.shape[1:]
        zt = z.view(B, T, h * w, D).permute(0, 2, 3, 1).reshape(B * h * w, D, T)
        zt = zt + self.temporal(zt)
        return zt.view(B, h, w, D, T).permute(0, 4, 1, 2, 3)      # [B, T, h, w, D]

    def encode(self, video):
        return self.image.vq.encode(self._latent(video))

    def decode(self, codes):                                     # [B, T, h, w]
        B, T = codes.shape[:2]
        return self.image.decode(codes.flatten(0, 1)).view(B, T, *self.image.decode(codes[:1, 0]).shape[1:])

    def forward(self, video):
        zq, codes, vq_loss = self.image.vq(self._latent(video))
        B, T = video.shape[:2]
        rec = self.image.dec(zq.flatten(0, 1).permute(0, 3, 1, 2)).view_as(video)
        return rec, codes, F.mse_loss(rec, video) + vq_loss


class AudioVQ(nn.Module):
    def __init__(self, n_mels: int = 80, dim: int = 256, code_dim: int = 64, codebook_size: int = 8192,
                 sample_rate: int = 16000, stride: int = 2):
        super().__init__()
        self.mel = MelFrontend(n_mels=n_mels, out_dim=dim, sr=sample_rate)
        self.enc = nn.Sequential(nn.Conv1d(dim, dim, 3, stride, 1), nn.SiLU(), nn.Conv1d(dim, code_dim, 1))
        self.vq = VectorQuantizer(codebook_size, code_dim)
        # codes -> log-mel frames (the input of MelVocoder); `stride` frames per code
        self.dec = nn.Sequential(nn.ConvTranspose1d(code_dim, dim, stride, stride), nn.SiLU(),
                                 nn.Conv1d(dim, n_mels, 3, padding=1))

    def _latent(self, wav):
        return self.enc(self.mel(wav).transpose(1, 2)).transpose(1, 2)    # [B, frames', D]

    def encode(self, wav):
        return self.vq.encode(self._latent(wav))

    def forward(self, wav):
        zq, codes, loss = self.vq(self._latent(wav))
        return zq, codes, loss

    def decode(self, codes: torch.Tensor) -> torch.Tensor:
        """codes [B, n] -> log-mel frames [B, n * stride, n_mels]."""
        z = self.vq.codebook.weight[codes]                               # [B, n, code_dim]
        return self.dec(z.transpose(1, 2)).transpose(1, 2)

    def reconstruction_loss(self, wav: torch.Tensor) -> torch.Tensor:
        """Codebook / commitment loss + L1 between the decoded and the input log-mel frames."""
        zq, codes, vq_loss = self.vq(self._latent(wav))
        mel = self.mel.mel(wav)
        rec = self.dec(zq.transpose(1, 2)).transpose(1, 2)
        n = min(rec.shape[1], mel.shape[1])
        return vq_loss + F.l1_loss(rec[:, :n], mel[:, :n])


class MelVocoder(nn.Module):
    """mel [B, frames, n_mels] -> waveform [B, frames * hop]; upsampling factors multiply to `hop`."""

    def __init__(self, n_mels: int = 80, width: int = 256, ups: tuple = (8, 8, 4)):
        super().__init__()
        layers = [nn.Conv1d(n_mels, width, 7, padding=3)]
        c = width
        for u in ups:
            layers += [nn.LeakyReLU(0.1), nn.ConvTranspose1d(c, c // 2, 2 * u, u, padding=u // 2)]
            c //= 2
        layers += [nn.LeakyReLU(0.1), nn.Conv1d(c, 1, 7, padding=3), nn.Tanh()]
        self.net = nn.Sequential(*layers)
        self.hop = 1
        for u in ups:
            self.hop *= u

    def forward(self, mel):
        return self.net(mel.transpose(1, 2)).squeeze(1)
