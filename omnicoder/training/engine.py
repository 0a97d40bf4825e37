"""Training step engine: forward, backward, gradient synchronisation, optimiser.

`Trainer.step(ids, labels)` is the public per-step API used by the pretraining
entry point, the benchmark and the tests.  With a process group it runs the
expert-parallel x data-parallel layout of :mod:`omnicoder.parallel` (experts
sharded over the EP group, dense parameters replicated with ZeRO-1 sharded
AdamW state); without one it is the single-device trainer.

The reference trainer's step (src/omnicoder/training/pretrain.py:915-952:
scaled backward, optimizer.step, zero_grad) has no gradient synchronisation at
all; it runs in a single process.
"""
from __future__ import annotations

import time
from dataclasses import dataclass

import torch

from ..config import ModelConfig, TrainConfig
from ..models.lm import OmniLM
from ..ops import FusedAdamW, cosine_lr


@dataclass
class StepStats:
    loss: torch.Tensor       # device scalar (no host sync)
    ce: torch.Tensor
    aux: torch.Tensor
    tokens: int
    lr: float


class Trainer:
    def __init__(self, model: OmniLM, tcfg: TrainConfig, parallel=None):
        self.model = model
        self.tcfg = tcfg
        self.parallel = parallel
        self.step_idx = 0
        if parallel is not None:
            self.opt = parallel.make_optimizer(model, tcfg)
        else:
            self.opt = FusedAdamW(model.parameters(), lr=tcfg.lr, betas=tuple(tcfg.betas), eps=tcfg.eps,
                                  weight_decay=tcfg.weight_decay, max_grad_norm=tcfg.grad_clip)
        model.set_aux_grad_scale(1.0 / max(1, tcfg.grad_accum))

    def lr_at(self, step: int) -> float:
        t = self.tcfg
        return cosine_lr(step, t.lr, t.warmup_steps, t.max_steps)

    def step(self, ids: torch.Tensor, labels: torch.Tensor, assume_all_valid: bool = False) -> StepStats:
        """One optimiser step over micro-batches `ids`/`labels` [B, S] (split into
        grad_accum chunks along the batch)."""
        accum = max(1, self.tcfg.grad_accum)
        chunks_ids = ids.chunk(accum, dim=0)
        chunks_lab = labels.chunk(accum, dim=0)
        loss_sum = ce_sum = aux_sum = None
        for mi, (ci, cl) in enumerate(zip(chunks_ids, chunks_lab)):
            if self.parallel is not None:
                self.parallel.before_forward(mi, len(chunks_ids))
            out = self.model(ci, labels=cl, assume_all_valid=assume_all_valid)
            loss = out["loss"] / accum
            loss.backward()
            l, c, a = out["loss"].detach(), out["ce"].detach(), out["aux"].detach()
            loss_sum = l if loss_sum is None else loss_sum + l
            ce_sum = c if ce_sum is None else ce_sum + c
            aux_sum = a if aux_sum is None else aux_sum + a
        lr = self.lr_at(self.step_idx)
        if self.parallel is not None:
            self.parallel.sync_and_step(self.model, self.opt, lr)
        else:
            self.opt.step(lr=lr)
        self.opt.zero_grad(set_to_none=True)
        self.step_idx += 1
        return StepStats(loss_sum / accum, ce_sum / accum, aux_sum / accum, ids.numel(), lr)

    # ------------------------------------------------------------------
    def state_dict(self) -> dict:
        return {"step": self.step_idx, "optimizer": self.opt.state_dict()}

    def load_state_dict(self, sd: dict):
        self.step_idx = int(sd["step"])
        self.opt.load_state_dict(sd["optimizer"])


def synthetic_batch(batch: int, seq: int, vocab: int, seed: int, step: int, device="cpu", pin: bool = False):
    """Uniform random token ids (labels = ids shifted left by one, last label from the
    same stream).  Deterministic in (seed, step)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed * 1_000_003 + step)
    stream = torch.randint(0, vocab, (batch, seq + 1), generator=g)
    ids, labels = stream[:, :-1].contiguous(), stream[:, 1:].contiguous()
    if pin:
        ids, labels = ids.pin_memory(), labels.pin_memory()
    if str(device) != "cpu":
        ids, labels = ids.to(device, non_blocking=True), labels.to(device, non_blocking=True)
    return ids, labels
