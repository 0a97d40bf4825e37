"""More task trainers: branch-train-merge upcycling, 3D latent, temporal video,
super-resolution, retention / write policies, reconstruction losses
(reference src/omnicoder/training/btm_upcycle.py, latent3d_train.py,
video_temporal_train.py, sr_train.py, retention_train.py, write_policy_train.py,
flow_recon.py).

btm_merge              branch-train-merge: the routed experts of several domain models fill the
                       student's expert slots round-robin (slot e <- domain e % n, that domain's
                       expert (e // n) % E_d); every other tensor (attention, norms, embeddings,
                       shared experts, routers) is the mean over the domains
train_latent3d         voxel head + orthographic renderer fitted to target images from the
                       language model's final hidden states (the reference feeds a zero
                       placeholder instead of hidden states, latent3d_train.py:46)
train_video_temporal   next-frame feature prediction with a causal temporal mixer, plus an
                       optional smoothness penalty on consecutive predictions
SuperResolver,         a sub-pixel convolution upscaler and its L1 / MSE training loop
train_super_resolution
retention_targets,     per-position keep scores (1 inside the recent window, a linear ramp over
train_policy_head      the older prefix) and a BCE trainer for a per-token policy head on the
                       model's hidden states (retention or write marks)
recon_loss             mse | mae | huber | feature (L1 between features of a frozen extractor)
"""
from __future__ import annotations

from typing import Callable, Iterable

import torch
import torch.nn as nn
import torch.nn.functional as F


# ----------------------------------------------------------------------------
# Branch-train-merge
# ----------------------------------------------------------------------------
@torch.no_grad()
def btm_merge(student: nn.Module, domains: list[nn.Module], expert_suffixes=(".ffn.w13", ".ffn.w2")) -> dict:
    """Fill `student` (same architecture family) from `domains`; returns {tensor name: source}."""
    if not domains:
        raise ValueError("btm_merge needs at least one domain model")
    dsd = [d.state_dict() for d in domains]
    report = {}
    for name, t in student.state_dict().items():
        srcs = [sd[name] for sd in dsd if name in sd]
        if not srcs:
            report[name] = "kept"
            continue
        if name.endswith(expert_suffixes) and t.dim() == 3:
            n = len(domains)
            for e in range(t.shape[0]):
                d = e % n
                src = dsd[d][name]
                j = (e // n) % src.shape[0]
                if src.shape[1:] != t.shape[1:]:
                    raise ValueError(f"{name}: expert shapes differ ({tuple(src.shape[1:])} vs {tuple(t.shape[1:])})")
                t[e].copy_(src[j])
            report[name] = "experts round-robin"
        elif all(s.shape == t.shape for s in srcs):
            t.copy_(torch.stack([s.float() for s in srcs]).mean(0).to(t.dtype))
            report[name] = f"mean of {len(srcs)}"
        else:
            report[name] = "kept (shape mismatch)"
    return report


# ----------------------------------------------------------------------------
# 3D latent
# ----------------------------------------------------------------------------
def train_latent3d(lm, head: nn.Module, renderer: nn.Module, batches: Iterable, steps: int, lr: float = 1e-3,
                   train_lm: bool = False) -> list[float]:
    """batches yield (ids [B, S], target images [B, 3, H, W] in [0, 1])."""
    params = list(head.parameters()) + list(renderer.parameters()) + (list(lm.parameters()) if train_lm else [])
    opt = torch.optim.AdamW(params, lr=lr)
    it, losses = iter(batches), []
    for _ in range(steps):
        ids, target = next(it)
        with torch.set_grad_enabled(train_lm):
            h, _ = lm.hidden(ids)
        h = h.view(ids.shape[0], ids.shape[1], -1).float()
        img = renderer(head(h))
        loss = F.mse_loss(img, target)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
    return losses


# ----------------------------------------------------------------------------
# Temporal video
# ----------------------------------------------------------------------------
def train_video_temporal(mixer: nn.Module, clips: Iterable, steps: int, lr: float = 1e-3,
                         smoothness: float = 0.0) -> list[float]:
    """clips yield frame features x [B, T, C]; `mixer` must be causal (its output at t sees
    frames <= t) and is trained to predict x[:, t + 1] from its output at t."""
    opt = torch.optim.AdamW(mixer.parameters(), lr=lr)
    it, losses = iter(clips), []
    for _ in range(steps):
        x = next(it)
        y = mixer(x)
        loss = F.mse_loss(y[:, :-1], x[:, 1:])
        if smoothness > 0:
            loss = loss + smoothness * (y[:, 1:] - y[:, :-1]).pow(2).mean()
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
    return losses


# ----------------------------------------------------------------------------
# Super-resolution
# ----------------------------------------------------------------------------
class SuperResolver(nn.Module):
    """low-res [B, 3, h, w] -> [B, 3, h * scale, w * scale]: convolutions, sub-pixel shuffle,
    plus the bilinear upsample of the input as a skip path."""

    def __init__(self, scale: int = 2, width: int = 32, depth: int = 3):
        super().__init__()
        self.scale = scale
        layers, c = [], 3
        for _ in range(depth):
            layers += [nn.Conv2d(c, width, 3, padding=1), nn.GELU()]
            c = width
        layers.append(nn.Conv2d(c, 3 * scale * scale, 3, padding=1))
        self.body = nn.Sequential(*layers)

    def forward(self, x):
        skip = F.interpolate(x, scale_factor=self.scale, mode="bilinear", align_corners=False)
        return skip + F.pixel_shuffle(self.body(x), self.scale)


def train_super_resolution(model: nn.Module, pairs: Iterable, steps: int, lr: float = 1e-3,
                           loss: str = "l1") -> list[float]:
    """pairs yield (low-res, high-res) image batches."""
    opt = torch.optim.AdamW(model.parameters(), lr=lr)
    fn = F.l1_loss if loss == "l1" else F.mse_loss
    it, losses = iter(pairs), []
    for _ in range(steps):
        lr_img, hr_img = next(it)
        l = fn(model(lr_img), hr_img)
        opt.zero_grad(set_to_none=True)
        l.backward()
        opt.step()
        losses.append(float(l.detach()))
    return losses


# ----------------------------------------------------------------------------
# Retention / write policies
# ----------------------------------------------------------------------------
def retention_targets(seq_len: int, window: int, device=None) -> torch.Tensor:
    """[seq_len] keep scores: 1 for the last `window` positions, rising linearly from 0 over
    the older prefix."""
    t = torch.zeros(seq_len, device=device)
    old = max(0, seq_len - window)
    if old > 0:
        t[:old] = torch.linspace(0.0, 1.0, old + 1, device=device)[:-1]
    t[old:] = 1.0
    return t


def train_policy_head(lm, head: nn.Module, batches: Iterable, steps: int, lr: float = 1e-3,
                      target_fn: Callable | None = None) -> list[float]:
    """batches yield ids [B, S] and, unless `target_fn(ids)` builds them, per-token targets
    [B, S] in [0, 1]; the head maps hidden states [B, S, D] to logits [B, S] (or [B, S, 1])."""
    opt = torch.optim.AdamW(head.parameters(), lr=lr)
    it, losses = iter(batches), []
    for _ in range(steps):
        item = next(it)
        ids, target = (item, target_fn(item)) if target_fn is not None else item
        with torch.no_grad():
            h, _ = lm.hidden(ids)
        logits = head(h.view(ids.shape[0], ids.shape[1], -1).float()).reshape(ids.shape)
        loss = F.binary_cross_entropy_with_logits(logits, target.float().expand_as(logits))
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
    return losses


# ----------------------------------------------------------------------------
# Reconstruction losses
# ----------------------------------------------------------------------------
def recon_loss(pred: torch.Tensor, target: torch.Tensor, kind: str = "mse", features: nn.Module | None = None,
               huber_delta: float = 1.0) -> torch.Tensor:
    if kind == "mse":
        return F.mse_loss(pred, target)
    if kind == "mae":
        return F.l1_loss(pred, target)
    if kind == "huber":
        return F.huber_loss(pred, target, delta=huber_delta)
    if kind == "feature":
        if features is None:
            raise ValueError("feature loss needs a feature extractor")
        with torch.no_grad():
            ft = features(target)
        return F.l1_loss(features(pred), ft)
    raise ValueError(f"unknown reconstruction loss {kind!r}")
