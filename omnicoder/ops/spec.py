"""Speculative-decoding verify step: per-sequence acceptance, next token and cache lengths.

`spec_verify` runs the sm_100a kernel (omnicoder/csrc/spec_verify.cu) on CUDA
tensors and the torch restatement below elsewhere; both follow the same rule:

  greedy (temperature <= 0): draft token j is accepted while it equals the target's
    argmax at position j; the next token is the target's argmax at the first
    rejected position (or at k when every draft token was accepted).
  sampling: p_t = softmax(logits / T); token j is accepted while
    u[j] < min(1, p_t(d_j) / p_d(d_j)); the next token is drawn by inverse CDF with
    u[k] from normalize(max(0, p_t - p_d)) at the first rejection, else from p_t at k.
  new_len = base_len + n_acc + 1.

Top-k / top-p filtered sampling is not part of the kernel; callers with filters use
the torch path of omnicoder.inference.generate.
"""
from __future__ import annotations

import torch

from . import _ext


def _inverse_cdf(w: torch.Tensor, u: float) -> int:
    """Smallest index whose inclusive prefix sum of w exceeds u * sum(w) (float64)."""
    w = w.double().clamp_min(0)
    c = torch.cumsum(w, 0)
    tot = float(c[-1])
    if tot <= 0:
        return 0
    idx = int(torch.searchsorted(c, torch.tensor([u * tot], dtype=torch.float64), right=True)[0])
    if idx >= w.numel():                       # rounding past the end: the last positive weight
        idx = int(torch.nonzero(w > 0)[-1])
    return idx


def spec_verify_torch(logits, pdraft, draft, u, base_len, temperature: float):
    """Restatement of the verify kernel with torch ops (reference and CPU path)."""
    B, K1, V = logits.shape
    K = K1 - 1
    n_acc = torch.empty(B, dtype=torch.int32)
    nxt = torch.empty(B, dtype=draft.dtype)
    for b in range(B):
        if temperature <= 0:
            am = logits[b].float().argmax(-1)
            j = 0
            while j < K and int(am[j]) == int(draft[b, j]):
                j += 1
            n_acc[b], nxt[b] = j, int(am[j])
            continue
        pt = torch.softmax(logits[b].double() / temperature, -1)
        j = 0
        while j < K:
            d = int(draft[b, j])
            ratio = float(pt[j, d]) / max(float(pdraft[b, j, d]), 1e-20)
            if not float(u[b, j]) < min(1.0, ratio):
                break
            j += 1
        w = (pt[j] - pdraft[b, j].double()).clamp_min(0) if j < K else pt[j]
        n_acc[b], nxt[b] = j, _inverse_cdf(w, float(u[b, K]))
    dev = logits.device
    n_acc, nxt = n_acc.to(dev), nxt.to(dev)
    return n_acc, nxt, base_len + (n_acc + 1).to(base_len.dtype)


def spec_verify(logits: torch.Tensor, pdraft: torch.Tensor | None, draft: torch.Tensor, u: torch.Tensor | None,
                base_len: torch.Tensor, temperature: float):
    """logits [B, K+1, V] of the target at the verified positions, pdraft [B, K, V] the draft's
    sampling distributions (None when greedy), draft [B, K] proposed ids, u [B, K+1] uniforms
    (None when greedy), base_len [B] cache lengths before the step.
    Returns (n_acc [B] int32, next token [B], new cache lengths [B])."""
    if logits.is_cuda:
        C = _ext.load()
        return C.spec_verify(logits.float().contiguous(), None if pdraft is None else pdraft.float().contiguous(),
                             draft.contiguous(), None if u is None else u.float().contiguous(), base_len.contiguous(),
                             float(temperature))
    return spec_verify_torch(logits, pdraft, draft, u, base_len, temperature)
