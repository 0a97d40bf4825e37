"""Causal (optionally windowed) multi-head attention with MLA / GQA key layouts.

Token-major layout, sequences of length S packed back to back (T = B * S):
  q       [T, H, Dq]                   Dq = Dk (+ Dr for MLA)
  k       [T, Hk, Dk]                  may be a strided view (MLA: into the kv up-projection)
  k_rope  [T, Dr] or None              MLA: rope part of the key, shared by all heads
  v       [T, Hk, Dv]                  may be a strided view
  out     [T, H, Dv]
GQA: query head h reads kv head h // (H // Hk).  Scale defaults to 1/sqrt(Dq).
`window` > 0 limits each query to the last `window` keys (itself included).
`mem_k`/`mem_v` ([B, M, H, Dq] / [B, M, H, Dv]) are memory slots every query of
sequence b may attend to, before the causal part.

On CUDA this runs the hand-written tcgen05 flash-attention kernels
(forward: S and O accumulators in TMEM, online softmax in registers; backward:
a dK/dV kernel and a dQ kernel, both recomputing P from the saved row
log-sum-exp).  On CPU it runs the dense masked softmax below, which is also the
oracle of the kernels.

The reference's prefill attention is not causal full attention (it attends to
8 landmark zeros, M memory slots and the last 16 padded rows;
src/omnicoder/modeling/attention.py:1135-1262); the compat model family keeps
that behaviour, this op implements exact causal/windowed attention.
"""
from __future__ import annotations

import math

import torch

from . import _ext


def _full_k(k: torch.Tensor, k_rope: torch.Tensor | None, H: int) -> torch.Tensor:
    if k_rope is None:
        return k
    Hk = k.shape[1]
    kr = k_rope.unsqueeze(1).expand(k.shape[0], Hk, k_rope.shape[-1])
    return torch.cat([k, kr], dim=-1)


def attention_torch(q, k, v, k_rope=None, *, seq: int, causal=True, window=0, scale=None, mem_k=None, mem_v=None,
                    return_lse=False):
    T, H, Dq = q.shape
    B = T // seq
    kf = _full_k(k, k_rope, H)
    Hk = kf.shape[1]
    rep = H // Hk
    qb = q.reshape(B, seq, H, Dq).transpose(1, 2).float()
    kb = kf.reshape(B, seq, Hk, Dq).transpose(1, 2).float()
    vb = v.reshape(B, seq, Hk, v.shape[-1]).transpose(1, 2).float()
    if rep > 1:
        kb = kb.repeat_interleave(rep, dim=1)
        vb = vb.repeat_interleave(rep, dim=1)
    sc = scale if scale is not None else 1.0 / math.sqrt(Dq)
    s = torch.matmul(qb, kb.transpose(-1, -2)) * sc
    i = torch.arange(seq, device=q.device)
    mask = torch.zeros(seq, seq, dtype=torch.bool, device=q.device)
    if causal:
        mask |= i[None, :] > i[:, None]
    if window > 0:
        mask |= i[None, :] <= i[:, None] - window
    s = s.masked_fill(mask, float("-inf"))
    if mem_k is not None:
        mk = mem_k.transpose(1, 2).float()  # [B, H, M, Dq]
        mv = mem_v.transpose(1, 2).float()
        sm = torch.matmul(qb, mk.transpose(-1, -2)) * sc
        s = torch.cat([sm, s], dim=-1)
        vb = torch.cat([mv, vb], dim=-2)
    lse = torch.logsumexp(s, dim=-1)
    p = torch.softmax(s, dim=-1)
    o = torch.matmul(p, vb)
    out = o.transpose(1, 2).reshape(T, H, -1).to(q.dtype)
    if return_lse:
        return out, lse
    return out


class _FlashAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, k_rope, seq, causal, window, scale):
        C = _ext.load()
        o, lse = C.attn_fwd(q, k, v, k_rope, seq, causal, window, scale)
        ctx.save_for_backward(q, k, v, k_rope if k_rope is not None else torch.empty(0, device=q.device), o, lse)
        ctx.has_rope = k_rope is not None
        ctx.cfg = (seq, causal, window, scale)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, k_rope, o, lse = ctx.saved_tensors
        seq, causal, window, scale = ctx.cfg
        C = _ext.load()
        grads = C.attn_bwd(q, k, v, k_rope if ctx.has_rope else None, o, lse, do.contiguous(), seq, causal, window,
                           scale)
        dk_rope = grads[3] if ctx.has_rope else None
        return grads[0], grads[1], grads[2], dk_rope, None, None, None, None


class _FlashAttnKVFn(torch.autograd.Function):
    """Attention whose keys and values are the two column blocks of one tensor kv
    [T, Hk, dk + dv] (the MLA key/value up-projection).  Backward writes dK and dV
    straight into one gradient of kv, so autograd adds no zero-filled slice gradients."""

    @staticmethod
    def forward(ctx, q, kv, dk, k_rope, seq, causal, window, scale):
        C = _ext.load()
        k, v = kv[:, :, :dk], kv[:, :, dk:]
        o, lse = C.attn_fwd(q, k, v, k_rope, seq, causal, window, scale)
        ctx.save_for_backward(q, kv, k_rope if k_rope is not None else torch.empty(0, device=q.device), o, lse)
        ctx.has_rope = k_rope is not None
        ctx.cfg = (dk, seq, causal, window, scale)
        return o

    @staticmethod
    def backward(ctx, do):
        q, kv, k_rope, o, lse = ctx.saved_tensors
        dk, seq, causal, window, scale = ctx.cfg
        C = _ext.load()
        dkv = torch.empty_like(kv)
        grads = C.attn_bwd(q, kv[:, :, :dk], kv[:, :, dk:], k_rope if ctx.has_rope else None, o, lse, do.contiguous(),
                           seq, causal, window, scale, None, dkv[:, :, :dk], dkv[:, :, dk:])
        return grads[0], dkv, None, (grads[3] if ctx.has_rope else None), None, None, None, None


def attention_kv(q: torch.Tensor, kv: torch.Tensor, dk: int, k_rope: torch.Tensor | None = None, *, seq: int,
                 causal: bool = True, window: int = 0, scale: float | None = None) -> torch.Tensor:
    """attention(q, kv[..., :dk], kv[..., dk:], k_rope) with a single gradient for kv."""
    sc = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if not q.is_cuda:
        return attention_torch(q, kv[:, :, :dk], kv[:, :, dk:], k_rope, seq=seq, causal=causal, window=window, scale=sc)
    return _FlashAttnKVFn.apply(q, kv, dk, k_rope, seq, causal, window, sc)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_rope: torch.Tensor | None = None, *, seq: int,
              causal: bool = True, window: int = 0, scale: float | None = None, mem_k=None, mem_v=None):
    sc = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if not q.is_cuda or mem_k is not None:
        if q.is_cuda:
            _ext.load()
        return attention_torch(q, k, v, k_rope, seq=seq, causal=causal, window=window, scale=sc, mem_k=mem_k,
                               mem_v=mem_v)
    return _FlashAttnFn.apply(q, k, v, k_rope, seq, causal, window, sc)
