"""Multimodal and verifier trainers (reference src/omnicoder/training/
verifier_distill.py, verifier_train.py and the omni/training/ modality
trainers: VQ codebooks, cross-modal alignment, vision-language pretraining).

train_vq(model, batches, steps)              image / video / audio VQ-VAE (reconstruction + VQ loss)
train_alignment(verifier, pairs, steps)      CrossModalVerifier contrastive (InfoNCE) training
vl_pretrain_step(lm, composer, opt, ...)     next-token loss on a [image tokens | text] sequence built
                                             by the MultimodalComposer from VQ codes
train_verifier_head(lm, head, batches, ...)  a verifier head on frozen hidden states: binary
                                             correctness targets (BCE) or KD to teacher scores (MSE)
"""
from __future__ import annotations

from typing import Callable, Iterable

import torch
import torch.nn as nn
import torch.nn.functional as F


def train_vq(model: nn.Module, batches: Iterable, steps: int, lr: float = 2e-4) -> list[float]:
    opt = torch.optim.AdamW(model.parameters(), lr=lr)
    out, it = [], iter(batches)
    for _ in range(steps):
        x = next(it)
        _, _, loss = model(x)
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        out.append(float(loss.detach()))
    return out


def train_alignment(verifier: nn.Module, pairs: Iterable, steps: int, lr: float = 1e-3,
                    modalities: tuple = ("text", "image")) -> list[float]:
    opt = torch.optim.AdamW(verifier.parameters(), lr=lr)
    out, it = [], iter(pairs)
    ma, mb = modalities
    for _ in range(steps):
        a, b = next(it)
        loss = verifier.loss(ma, a, mb, b)
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        out.append(float(loss.detach()))
    return out


def vl_pretrain_step(lm, composer, opt, image_codes: torch.Tensor, text_ids: torch.Tensor) -> float:
    """One step of next-token prediction over [image tokens, text] (loss on the text part)."""
    seq = composer.fuse_codes(text_ids, image=image_codes.reshape(image_codes.shape[0], -1))
    labels = seq.clone()
    labels[:, :seq.shape[1] - text_ids.shape[1]] = -100
    loss = lm(seq[:, :-1], labels=labels[:, 1:])["loss"]
    loss.backward()
    opt.step()
    opt.zero_grad(set_to_none=True)
    return float(loss.detach())


class VerifierHead(nn.Module):
    """Scores a (prompt, answer) sequence from its last hidden state."""

    def __init__(self, d_model: int):
        super().__init__()
        self.net = nn.Sequential(nn.Linear(d_model, d_model // 2), nn.GELU(), nn.Linear(d_model // 2, 1))

    def forward(self, hidden_last: torch.Tensor) -> torch.Tensor:
        return self.net(hidden_last.float()).squeeze(-1)


def train_verifier_head(lm, head: VerifierHead, batches: Iterable, steps: int, lr: float = 1e-3,
                        teacher: Callable | None = None) -> list[float]:
    """batches yield (ids [B, S], targets [B] in {0, 1}); with `teacher`, targets are replaced by
    teacher(ids) scores in [0, 1] and the head is fitted by MSE on the logits' sigmoid."""
    opt = torch.optim.AdamW(head.parameters(), lr=lr)
    out, it = [], iter(batches)
    for _ in range(steps):
        ids, tgt = next(it)
        with torch.no_grad():
            h, _ = lm.hidden(ids)
            last = h.view(ids.shape[0], ids.shape[1], -1)[:, -1]
        logits = head(last)
        if teacher is not None:
            loss = F.mse_loss(torch.sigmoid(logits), teacher(ids).float())
        else:
            loss = F.binary_cross_entropy_with_logits(logits, tgt.float())
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        out.append(float(loss.detach()))
    return out
