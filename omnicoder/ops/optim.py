"""Fused AdamW with fp32 master weights (bf16 model parameters).

One sm_100a kernel per parameter updates the fp32 master copy, the two moment
buffers and writes the bf16 parameter, reading the bf16 gradient once.  An
optional global-norm clip is computed on the device (no host synchronisation):
each gradient's squared norm accumulates into one device scalar that the update
kernels read.  The update rule is torch.optim.AdamW's (decoupled weight decay,
bias-corrected moments), the optimiser the reference trainer uses
(src/omnicoder/training/pretrain.py:582).
"""
from __future__ import annotations

import math
from typing import Iterable

import torch

from . import _ext


class FusedAdamW:
    SMALL = 1 << 20   # elements: parameters up to this size are updated by the multi-tensor kernels

    def __init__(self, params: Iterable[torch.nn.Parameter], lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, max_grad_norm: float = 0.0, no_decay_1d: bool = True):
        self.params = [p for p in params if p.requires_grad]
        self.lr = lr
        self.betas = betas
        self.eps = eps
        self.weight_decay = weight_decay
        self.max_grad_norm = max_grad_norm
        self.no_decay_1d = no_decay_1d
        self.step_count = 0
        self.state: dict[int, dict[str, torch.Tensor]] = {}
        for i, p in enumerate(self.params):
            master = p.detach().float().clone() if p.dtype != torch.float32 else p.detach()
            self.state[i] = {"master": master, "m": torch.zeros_like(master), "v": torch.zeros_like(master)}
        self._norm = None

    # ------------------------------------------------------------------
    def zero_grad(self, set_to_none: bool = True):
        for p in self.params:
            if set_to_none:
                p.grad = None
            elif p.grad is not None:
                p.grad.zero_()

    def _wd(self, p):
        return 0.0 if (self.no_decay_1d and p.dim() <= 1) else self.weight_decay

    @torch.no_grad()
    def step(self, lr: float | None = None, grad_scale: float = 1.0):
        if lr is not None:
            self.lr = lr
        self.step_count += 1
        t = self.step_count
        b1, b2 = self.betas
        # the kernels below write the parameters in place without moving their version
        # counters: quantised weight copies (fp8 projections) are redone after this step
        from .fp8 import WEIGHTS
        WEIGHTS.bump()
        cuda = len(self.params) > 0 and self.params[0].is_cuda
        if cuda:
            C = _ext.load()
            grads = {i: (p.grad if p.grad.dtype == torch.bfloat16 else p.grad.to(torch.bfloat16)).contiguous()
                     for i, p in enumerate(self.params) if p.grad is not None}
            # parameters up to SMALL elements (norm weights, routers) go through the multi-tensor
            # kernels, a few launches for all of them instead of two per parameter
            small = [i for i in grads if self.params[i].numel() <= self.SMALL]
            large = [i for i in grads if self.params[i].numel() > self.SMALL]
            norm = None
            if self.max_grad_norm > 0:
                if self._norm is None:
                    self._norm = torch.zeros(1, device=self.params[0].device, dtype=torch.float32)
                self._norm.zero_()
                C.sq_norm_multi([grads[i] for i in small], grad_scale, self._norm)
                for i in large:
                    C.sq_norm(grads[i], grad_scale, self._norm)
                norm = self._norm
            if small:
                pbs = [self.params[i].data if self.params[i].dtype == torch.bfloat16 else None for i in small]
                C.adamw_multi([self.state[i]["master"] for i in small], [self.state[i]["m"] for i in small],
                              [self.state[i]["v"] for i in small], [grads[i] for i in small], pbs,
                              [self._wd(self.params[i]) for i in small], self.lr, b1, b2, self.eps, t, grad_scale,
                              norm, self.max_grad_norm)
            for i in large:
                p, st = self.params[i], self.state[i]
                pb = p.data if p.dtype == torch.bfloat16 else None
                C.adamw(st["master"], st["m"], st["v"], grads[i], pb, self.lr, b1, b2, self.eps, self._wd(p), t,
                        grad_scale, norm, self.max_grad_norm)
            for i in grads:
                p, st = self.params[i], self.state[i]
                if p.dtype != torch.bfloat16 and p.data.data_ptr() != st["master"].data_ptr():
                    p.data.copy_(st["master"])
            return
        # CPU reference (identical update rule, fp32)
        clip = 1.0
        if self.max_grad_norm > 0:
            tot = sum(float((p.grad.float() * grad_scale).pow(2).sum()) for p in self.params if p.grad is not None)
            clip = min(1.0, self.max_grad_norm / (math.sqrt(tot) + 1e-6))
        bc1 = 1 - b1 ** t
        bc2 = 1 - b2 ** t
        for i, p in enumerate(self.params):
            if p.grad is None:
                continue
            st = self.state[i]
            g = p.grad.float() * (grad_scale * clip)
            m, v, w = st["m"], st["v"], st["master"]
            m.mul_(b1).add_(g, alpha=1 - b1)
            v.mul_(b2).addcmul_(g, g, value=1 - b2)
            w.mul_(1 - self.lr * self._wd(p))
            denom = (v.sqrt() / math.sqrt(bc2)).add_(self.eps)
            w.addcdiv_(m, denom, value=-self.lr / bc1)
            if p.data.data_ptr() != w.data_ptr():
                p.data.copy_(w)

    # ------------------------------------------------------------------
    def state_dict(self) -> dict:
        return {"step": self.step_count, "lr": self.lr, "betas": self.betas, "eps": self.eps,
                "weight_decay": self.weight_decay, "max_grad_norm": self.max_grad_norm,
                "state": {i: {k: v.detach().cpu() for k, v in s.items()} for i, s in self.state.items()}}

    def load_state_dict(self, sd: dict):
        self.step_count = int(sd["step"])
        self.lr = sd.get("lr", self.lr)
        for i, s in sd["state"].items():
            i = int(i)
            for k, v in s.items():
                self.state[i][k].copy_(v.to(self.state[i][k].device))
        for i, p in enumerate(self.params):
            p.data.copy_(self.state[i]["master"].to(p.dtype))


def cosine_lr(step: int, base_lr: float, warmup: int, total: int, min_ratio: float = 0.1) -> float:
    """Linear warmup then cosine decay to min_ratio * base_lr."""
    if warmup > 0 and step < warmup:
        return base_lr * (step + 1) / warmup
    if total <= warmup:
        return base_lr
    p = min(1.0, (step - warmup) / max(1, total - warmup))
    return base_lr * (min_ratio + (1 - min_ratio) * 0.5 * (1 + math.cos(math.pi * p)))
