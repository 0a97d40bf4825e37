"""Continuous audio-latent reconstruction (reference src/omnicoder/training/audio_recon.py:64-260 and
audio_latent_supervised.py: the model's audio latent head is trained to produce the latent an audio
encoder gives for a clip, with spectral side losses when raw waveforms are available).

  target:  MelPoolEncoder(wave) -> z [B, P, C]: log-mel frames pooled into P time segments and a fixed
           random projection to C channels (the stand-in when no pretrained audio codec is present;
           the projection is drawn once from a seed, so targets are a fixed function of the audio)
  predict: LatentQueryHead(LM state at the last prompt position) -> z_hat [B, P, C]
  loss  =  recon(z_hat, z)                                           (mse / mae / huber)
         + 0.1  * |proj_mel(mean_P z_hat)  - time-mean mel|_1         (80 mel bands)
         + 0.05 * |proj_stft(mean_P z_hat) - time-mean |STFT||_1      (n_fft 1024 -> 513 bins, hop 256)
With `flow=True` the head is trained by rectified flow on the same targets instead of the plain
reconstruction term (the trainer of omnicoder.training.flow_recon), and the side losses read the
clean-latent estimate x_t - t v_hat.
"""
from __future__ import annotations

import argparse
import json
import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .flow_recon import FlowReconTrainer, LatentQueryHead


class MelPoolEncoder(nn.Module):
    def __init__(self, segments: int = 4, channels: int = 16, n_mels: int = 80, sr: int = 16000, seed: int = 0):
        super().__init__()
        from ..multimodal.encoders import MelFrontend
        self.front = MelFrontend(n_mels=n_mels, out_dim=channels, sr=sr)
        self.segments = segments
        g = torch.Generator().manual_seed(seed)
        self.register_buffer("proj", torch.randn(n_mels, channels, generator=g) / math.sqrt(n_mels))

    @torch.no_grad()
    def log_mel(self, wav: torch.Tensor) -> torch.Tensor:
        """[B, samples] -> [B, frames, n_mels]."""
        return self.front.mel(wav.float())

    @torch.no_grad()
    def forward(self, wav: torch.Tensor) -> torch.Tensor:
        m = self.log_mel(wav)                                                      # [B, T, M]
        pooled = F.adaptive_avg_pool1d(m.transpose(1, 2), self.segments).transpose(1, 2)
        return pooled @ self.proj.to(pooled.device)                                # [B, P, C]


class AudioReconTrainer(FlowReconTrainer):
    def __init__(self, lm, head: LatentQueryHead, encoder: MelPoolEncoder, lr: float = 1e-3, flow: bool = False,
                 recon: str = "mse", train_lm: bool = False, mel_weight: float = 0.1, stft_weight: float = 0.05,
                 n_fft: int = 1024, hop: int = 256, refiner: nn.Module | None = None):
        C = head.mlp[-1].out_features
        n_mels = encoder.proj.shape[0]
        self.proj_mel = nn.Sequential(nn.LayerNorm(C), nn.Linear(C, 128), nn.GELU(), nn.Linear(128, n_mels))
        self.proj_stft = nn.Sequential(nn.LayerNorm(C), nn.Linear(C, 256), nn.GELU(), nn.Linear(256, n_fft // 2 + 1))
        dev = head.q.device
        self.proj_mel.to(dev)
        self.proj_stft.to(dev)
        super().__init__(lm, head, encoder, lr, flow, recon, train_lm, refiner=refiner)
        self.opt.add_param_group({"params": list(self.proj_mel.parameters()) + list(self.proj_stft.parameters())})
        self.mel_weight, self.stft_weight, self.n_fft, self.hop = mel_weight, stft_weight, n_fft, hop

    def loss(self, wav: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        wav = wav.to(ids.device).float()
        loss, z_hat = self.loss_and_estimate(self.enc(wav), self._state(ids))
        pooled = z_hat.mean(1)                                                     # [B, C]
        if self.mel_weight:
            mel = self.enc.log_mel(wav).mean(1)
            loss = loss + self.mel_weight * (self.proj_mel(pooled) - mel).abs().mean()
        if self.stft_weight:
            win = torch.hann_window(self.n_fft, device=wav.device)
            mag = torch.stft(wav, self.n_fft, self.hop, window=win, return_complex=True).abs().mean(-1)
            loss = loss + self.stft_weight * (self.proj_stft(pooled) - mag).abs().mean()
        return loss


def synthetic_tones(n: int, samples: int = 8000, sr: int = 16000, seed: int = 0) -> tuple[torch.Tensor, list[str]]:
    """n sine tones at distinct pitches with their captions."""
    g = torch.Generator().manual_seed(seed)
    t = torch.arange(samples) / sr
    freqs = 200 + 100 * torch.arange(n)
    waves = torch.stack([torch.sin(2 * math.pi * float(f) * t) * (0.5 + 0.5 * torch.rand((), generator=g))
                         for f in freqs])
    return waves, [f"a tone at {int(f)} hertz" for f in freqs]


def main(argv=None):
    from ..config import get_preset
    from ..models.lm import build_model
    from .tokenizer import get_tokenizer
    ap = argparse.ArgumentParser(description="audio latent reconstruction training")
    ap.add_argument("--preset", default="tiny_moe")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--segments", type=int, default=4)
    ap.add_argument("--latent_dim", type=int, default=16)
    ap.add_argument("--recon_loss", default="mse", choices=["mse", "mae", "huber"])
    ap.add_argument("--flow_loss", action="store_true")
    ap.add_argument("--mel_weight", type=float, default=0.1)
    ap.add_argument("--stft_weight", type=float, default=0.05)
    ap.add_argument("--use_refiner", action="store_true", help="train a latent refiner beside the head")
    ap.add_argument("--lr", type=float, default=1e-3)
    ap.add_argument("--out", default="weights/audio_recon_head.pt")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    dev = torch.device(a.device)
    lm = build_model(get_preset(a.preset), device=dev, dtype=torch.float32, seed=0).eval()
    head = LatentQueryHead(lm.cfg.d_model, a.segments, a.latent_dim).to(dev)
    enc = MelPoolEncoder(a.segments, a.latent_dim).to(dev)
    from ..multimodal.video import LatentRefiner
    refiner = LatentRefiner(a.latent_dim).to(dev) if a.use_refiner else None
    tr = AudioReconTrainer(lm, head, enc, a.lr, a.flow_loss, a.recon_loss, mel_weight=a.mel_weight,
                           stft_weight=a.stft_weight, refiner=refiner)
    tok = get_tokenizer(lm.cfg.vocab_size)
    waves, caps = synthetic_tones(8)
    g = torch.Generator().manual_seed(0)
    losses = []
    for _ in range(a.steps):
        idx = torch.randint(0, len(caps), (a.batch,), generator=g)
        enc_ids = [tok.encode(caps[int(i)]) for i in idx]
        L = max(len(e) for e in enc_ids)
        ids = torch.tensor([e + [0] * (L - len(e)) for e in enc_ids], device=dev)
        losses.append(tr.step(waves[idx].to(dev), ids))
    torch.save({"head": head.state_dict(), "proj_mel": tr.proj_mel.state_dict(),
                "proj_stft": tr.proj_stft.state_dict(), "flow": a.flow_loss,
                **({"refiner": refiner.state_dict()} if refiner is not None else {})}, a.out)
    print(json.dumps({"steps": a.steps, "first_loss": losses[0], "last_loss": losses[-1], "out": a.out}))
    return 0


if __name__ == "__main__":
    main()
