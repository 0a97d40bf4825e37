"""LM head + softmax cross entropy without materialising the full logits tensor.

CUDA: rows are processed in chunks; for each chunk the tcgen05 GEMM produces
bf16 logits, one kernel computes the row losses and overwrites the logits with
their gradient (softmax - onehot, scaled), and two more GEMMs produce the
hidden-state gradient and accumulate the head-weight gradient (fp32).  The
gradients are computed during forward, so backward only rescales them by the
incoming scalar.  Loss matches F.cross_entropy(reduction="mean") over the
labels that are not `ignore_index` (the reference's token loss,
src/omnicoder/training/pretrain.py:727), plus an optional z-loss
(z * mean(logsumexp^2)).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import _ext
from .gemm import mm_nn, mm_nt, mm_tn


class _HeadCEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w, labels, ignore_index, z_loss, chunk, assume_all_valid):
        C = _ext.load()
        h2 = h.reshape(-1, h.shape[-1]).contiguous()
        lab = labels.reshape(-1).contiguous().long()
        T = h2.shape[0]
        if assume_all_valid:
            n_valid = torch.full((), float(T), device=h.device)   # a fill kernel, no host copy
            scale = 1.0 / T
        else:
            lab = torch.where(lab == ignore_index, torch.full_like(lab, -1), lab)
            n_valid = (lab >= 0).sum().float().clamp_min(1.0)
            scale = 1.0
        dh = torch.empty_like(h2)
        dw32 = torch.zeros(w.shape, device=h.device, dtype=torch.float32)
        losses = torch.empty(T, device=h.device, dtype=torch.float32)
        for s in range(0, T, chunk):
            e = min(T, s + chunk)
            logits = mm_nt(h2[s:e], w)
            loss_rows, _ = C.cross_entropy(logits, lab[s:e], logits, scale, z_loss)
            losses[s:e] = loss_rows
            dh[s:e] = mm_nn(logits, w)
            mm_tn(logits, h2[s:e], accumulate_into=dw32)
        loss = losses.sum() / n_valid
        if not assume_all_valid:
            inv = 1.0 / n_valid
            dh.mul_(inv.to(dh.dtype))
            dw32.mul_(inv)
        ctx.save_for_backward(dh, dw32)
        ctx.shape = h.shape
        ctx.wdtype = w.dtype
        return loss

    @staticmethod
    def backward(ctx, g):
        dh, dw32 = ctx.saved_tensors
        dh = dh * g.to(dh.dtype)
        dw = (dw32 * g).to(ctx.wdtype)
        return dh.view(ctx.shape), dw, None, None, None, None, None


def lm_head_cross_entropy(h: torch.Tensor, w: torch.Tensor, labels: torch.Tensor, ignore_index: int = -100,
                          z_loss: float = 0.0, chunk: int = 8192, assume_all_valid: bool = False) -> torch.Tensor:
    """mean over valid labels of CE(h @ w.T, labels) (+ z_loss * mean(lse^2))."""
    if not h.is_cuda:
        logits = (h.reshape(-1, h.shape[-1]) @ w.t()).float()
        lab = labels.reshape(-1)
        loss = F.cross_entropy(logits, lab, ignore_index=ignore_index)
        if z_loss > 0:
            valid = lab != ignore_index
            lse = torch.logsumexp(logits, -1)
            loss = loss + z_loss * (lse[valid] ** 2).mean()
        return loss
    return _HeadCEFn.apply(h, w, labels, ignore_index, z_loss, chunk, assume_all_valid)


def cross_entropy_logits(logits: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    """Per-row loss of materialised logits (inference / evaluation)."""
    if not logits.is_cuda:
        return F.cross_entropy(logits.float(), labels.long(), reduction="none")
    lg = logits.reshape(-1, logits.shape[-1]).contiguous().to(torch.bfloat16)
    loss, _ = _ext.load().cross_entropy(lg, labels.reshape(-1).long().contiguous(), None, 1.0, 0.0)
    return loss
