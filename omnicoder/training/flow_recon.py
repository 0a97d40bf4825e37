"""Latent reconstruction / flow-matching training of the continuous image-latent head
(reference src/omnicoder/training/flow_recon.py: the language model produces continuous latent
tokens that match the latents an image encoder gives for the paired image, with a plain
reconstruction loss and optionally a flow / diffusion loss on noised latents).

  encoder(images [B, 3, S, S]) -> target latents z0 [B, P, C]   (P patch latents, or 1 pooled)
  lm.hidden(prompt ids)        -> h [B, D] at the last prompt position
  reconstruction:  LatentQueryHead(h) -> z_hat [B, P, C];  loss = recon_loss(z_hat, z0)  (mse / mae / huber)
  flow matching (rectified flow, `flow=True`):  t ~ logit-normal, x_t = (1 - t) z0 + t eps,
      the head predicts the velocity v = eps - z0 from (h, x_t, t);  loss = E[w(t) |v_hat - v|^2]
      with w(t) = 1 / (t^2 + (1 - t)^2) (the weighting that equalises the noise-prediction scale).
`sample()` integrates the learned velocity from noise (t = 1 -> 0, Euler) to a latent.
With a refiner (the reference's --use_refiner: a small residual MLP over latents), the refiner is
trained beside the head to map the head's estimate (detached) to the target, and `sample()` applies
it last; its weights go into the checkpoint under "refiner" (the latent-refine tool reads them).

`PatchPoolEncoder` is the stand-in encoder when no pretrained image autoencoder is available
(the reference's IdentityAdapter): average pooling to a P-patch grid and a fixed random projection
to C channels.
"""
from __future__ import annotations

import argparse
import json
import math

import torch
import torch.nn as nn
import torch.nn.functional as F


class PatchPoolEncoder(nn.Module):
    def __init__(self, grid: int = 4, channels: int = 16, seed: int = 0):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.grid = grid
        self.register_buffer("proj", torch.randn(3, channels, generator=g) / math.sqrt(3))

    @torch.no_grad()
    def forward(self, images: torch.Tensor) -> torch.Tensor:
        p = F.adaptive_avg_pool2d(images.float(), self.grid)                # [B, 3, g, g]
        return p.flatten(2).transpose(1, 2) @ self.proj.to(p.device)         # [B, g*g, C]


class LatentQueryHead(nn.Module):
    """P learned queries conditioned on the LM state h (and, for flow matching, on the noised latent
    and the time) -> P latent vectors."""

    def __init__(self, d_model: int, patches: int, channels: int, width: int = 256):
        super().__init__()
        self.q = nn.Parameter(torch.randn(patches, width) * 0.02)
        self.h_in = nn.Linear(d_model, width)
        self.x_in = nn.Linear(channels, width)
        self.t_in = nn.Linear(16, width)
        self.mlp = nn.Sequential(nn.LayerNorm(width), nn.Linear(width, 2 * width), nn.GELU(),
                                 nn.Linear(2 * width, channels))

    @staticmethod
    def _tfeat(t: torch.Tensor) -> torch.Tensor:
        f = torch.exp(torch.linspace(0, math.log(1000.0), 8, device=t.device))
        a = t[:, None] * f[None]
        return torch.cat([a.sin(), a.cos()], -1)                              # [B, 16]

    def forward(self, h: torch.Tensor, x_t: torch.Tensor | None = None, t: torch.Tensor | None = None):
        z = self.q[None] + self.h_in(h.float())[:, None]
        if x_t is not None:
            z = z + self.x_in(x_t.float()) + self.t_in(self._tfeat(t))[:, None]
        return self.mlp(z)


def _weight(t: torch.Tensor) -> torch.Tensor:
    return 1.0 / (t * t + (1 - t) ** 2)


class FlowReconTrainer:
    def __init__(self, lm, head: LatentQueryHead, encoder: nn.Module, lr: float = 1e-3, flow: bool = False,
                 recon: str = "mse", train_lm: bool = False, refiner: nn.Module | None = None):
        self.lm, self.head, self.enc, self.flow, self.recon = lm, head, encoder, flow, recon
        self.refiner = refiner
        params = list(head.parameters()) + ([p for p in lm.parameters() if p.requires_grad] if train_lm else [])
        params += list(refiner.parameters()) if refiner is not None else []
        self.train_lm = train_lm
        self.opt = torch.optim.AdamW(params, lr=lr)

    def _state(self, ids: torch.Tensor) -> torch.Tensor:
        ctx = torch.enable_grad() if self.train_lm else torch.no_grad()
        with ctx:
            y, _ = self.lm.hidden(ids)
        return y.view(ids.shape[0], ids.shape[1], -1)[:, -1]

    def loss_and_estimate(self, z0: torch.Tensor, h: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Loss for target latents z0 given LM states h, and the head's estimate of z0: its output
        (reconstruction) or x_t - t v_hat (flow: the clean latent the predicted velocity points to)."""
        from .multimodal_tasks import recon_loss
        if not self.flow:
            z_hat = self.head(h)
            loss = recon_loss(z_hat, z0, self.recon)
        else:
            B = z0.shape[0]
            t = torch.sigmoid(torch.randn(B, device=z0.device))                # logit-normal times
            eps = torch.randn_like(z0)
            x_t = (1 - t)[:, None, None] * z0 + t[:, None, None] * eps
            v = self.head(h, x_t, t)
            loss = (_weight(t)[:, None, None] * (v - (eps - z0)) ** 2).mean()
            z_hat = x_t - t[:, None, None] * v
        if self.refiner is not None:       # a post-processor of the head's estimate, trained beside it
            loss = loss + recon_loss(self.refiner(z_hat.detach()), z0, self.recon)
        return loss, z_hat

    def loss(self, images: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        return self.loss_and_estimate(self.enc(images).to(ids.device), self._state(ids))[0]

    def step(self, images: torch.Tensor, ids: torch.Tensor) -> float:
        loss = self.loss(images, ids)
        self.opt.zero_grad(set_to_none=True)
        loss.backward()
        self.opt.step()
        return float(loss.detach())

    @torch.no_grad()
    def sample(self, ids: torch.Tensor, steps: int = 16, seed: int = 0) -> torch.Tensor:
        """Latents for the prompts: the reconstruction head's output, or (flow) Euler integration of
        the learned velocity from noise at t = 1 to t = 0."""
        h = self._state(ids)
        if not self.flow:
            x = self.head(h)
        else:
            P, C = self.head.q.shape[0], self.head.mlp[-1].out_features
            g = torch.Generator(device=ids.device).manual_seed(seed)
            x = torch.randn(ids.shape[0], P, C, generator=g, device=ids.device)
            ts = torch.linspace(1.0, 0.0, steps + 1, device=ids.device)
            for i in range(steps):
                t = ts[i].expand(ids.shape[0])
                x = x + (ts[i + 1] - ts[i]) * self.head(h, x, t)               # dx/dt = v
        return self.refiner(x) if self.refiner is not None else x


def main(argv=None):
    from ..config import get_preset
    from ..models.lm import build_model
    from .tokenizer import get_tokenizer
    ap = argparse.ArgumentParser(description="latent reconstruction / flow-matching training")
    ap.add_argument("--preset", default="tiny_moe")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--image_size", type=int, default=32)
    ap.add_argument("--grid", type=int, default=4)
    ap.add_argument("--channels", type=int, default=16)
    ap.add_argument("--flow_loss", action="store_true")
    ap.add_argument("--recon_loss", default="mse", choices=["mse", "mae", "huber"])
    ap.add_argument("--use_refiner", action="store_true", help="train a latent refiner beside the head")
    ap.add_argument("--lr", type=float, default=1e-3)
    ap.add_argument("--out", default="weights/flow_recon_head.pt")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    dev = torch.device(a.device)
    lm = build_model(get_preset(a.preset), device=dev, dtype=torch.float32, seed=0).eval()
    head = LatentQueryHead(lm.cfg.d_model, a.grid * a.grid, a.channels).to(dev)
    from ..multimodal.video import LatentRefiner
    refiner = LatentRefiner(a.channels).to(dev) if a.use_refiner else None
    tr = FlowReconTrainer(lm, head, PatchPoolEncoder(a.grid, a.channels).to(dev), a.lr, a.flow_loss, a.recon_loss,
                          refiner=refiner)
    tok = get_tokenizer(lm.cfg.vocab_size)
    g = torch.Generator().manual_seed(0)
    colors = torch.rand(8, 3, generator=g)
    names = [f"a picture of colour {i}" for i in range(8)]
    losses = []
    for step in range(a.steps):
        idx = torch.randint(0, 8, (a.batch,), generator=g)
        imgs = colors[idx][:, :, None, None].expand(-1, -1, a.image_size, a.image_size).to(dev)
        enc = [tok.encode(names[int(i)]) for i in idx]
        L = max(len(e) for e in enc)
        ids = torch.tensor([e + [0] * (L - len(e)) for e in enc], device=dev)
        losses.append(tr.step(imgs, ids))
    torch.save({"head": head.state_dict(), "flow": a.flow_loss,
                **({"refiner": refiner.state_dict()} if refiner is not None else {})}, a.out)
    print(json.dumps({"steps": a.steps, "first_loss": losses[0], "last_loss": losses[-1], "out": a.out}))
    return 0


if __name__ == "__main__":
    main()
