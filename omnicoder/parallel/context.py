"""Context (sequence) parallel attention, all-to-all over heads ("Ulysses" layout).

The reference has no context parallelism; its long-context path is windowing,
memory slots, compressive KV and RoPE scaling
(src/omnicoder/modeling/attention.py:646-649, src/omnicoder/config.py:61-94).
This module adds it for long prefill / training sequences.

Layout in a group of W ranks: each of the B sequences (length S) is split into
W contiguous chunks of s = S / W tokens; rank r holds chunk r of every sequence,
token-major [B * s, heads, dim].  Attention:
  1. all-to-all: rank r sends head group j (H / W query heads, Hk / W kv heads)
     of its chunk to rank j and receives its own head group of every chunk, so it
     holds full sequences for H / W heads: [B * S, H / W, dim];
  2. the flash attention kernel over those full sequences (causal / windowed
     masks are exact, since every rank sees whole sequences);
  3. all-to-all back to the sequence-chunk layout.
The MLA shared rope key (one [T, Dr] row per token for all heads) travels as
one extra "head" per destination.  Both all-to-alls are autograd functions whose
backward is the inverse all-to-all.  One all_to_all_single per tensor and
direction: on NVSwitch every rank sends (W - 1) / W of its q, k, v and output
bytes, against the all-gather of full K / V that a ring schedule would need.

`shard_sequence` / `gather_sequence` convert [B, S, ...] batches to and from the
chunked layout; `positions` gives the RoPE positions of the local tokens.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops.attention import attention


def _a2a(x: torch.Tensor, group) -> torch.Tensor:
    x = x.contiguous()
    out = torch.empty_like(x)
    dist.all_to_all_single(out, x, group=group)
    return out


def _seq_to_head(x: torch.Tensor, B: int, W: int, group) -> torch.Tensor:
    """[B * s, W * h, d] (sequence chunk, all heads) -> [B * S, h, d] (full sequences, head group)."""
    Bs, Hh, d = x.shape
    s, h = Bs // B, Hh // W
    send = x.reshape(B, s, W, h, d).permute(2, 0, 1, 3, 4)              # [dst, B, s, h, d]
    recv = _a2a(send, group)                                            # [src chunk, B, s, h, d]
    return recv.permute(1, 0, 2, 3, 4).reshape(B * W * s, h, d)


def _head_to_seq(x: torch.Tensor, B: int, W: int, group) -> torch.Tensor:
    """[B * S, h, d] (full sequences, head group) -> [B * s, W * h, d] (sequence chunk, all heads)."""
    BS, h, d = x.shape
    s = BS // (B * W)
    send = x.reshape(B, W, s, h, d).permute(1, 0, 2, 3, 4)              # [dst chunk, B, s, h, d]
    recv = _a2a(send, group)                                            # [src head group, B, s, h, d]
    return recv.permute(1, 2, 0, 3, 4).reshape(B * s, W * h, d)


class _SeqToHead(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, B, W, group):
        ctx.cfg = (B, W, group)
        return _seq_to_head(x, B, W, group)

    @staticmethod
    def backward(ctx, g):
        B, W, group = ctx.cfg
        return _head_to_seq(g, B, W, group), None, None, None


class _HeadToSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, B, W, group):
        ctx.cfg = (B, W, group)
        return _head_to_seq(x, B, W, group)

    @staticmethod
    def backward(ctx, g):
        B, W, group = ctx.cfg
        return _seq_to_head(g, B, W, group), None, None, None


def context_parallel_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_rope: torch.Tensor | None = None,
                               *, batch: int, group=None, causal: bool = True, window: int = 0,
                               scale: float | None = None) -> torch.Tensor:
    """q [B * s, H, Dq], k [B * s, Hk, Dk], v [B * s, Hk, Dv], k_rope [B * s, Dr] or None, local
    chunks of `batch` sequences -> out [B * s, H, Dv].  H and Hk must be multiples of the group size."""
    group = group if group is not None else dist.group.WORLD
    W = dist.get_world_size(group)
    H, Hk = q.shape[1], k.shape[1]
    if H % W or Hk % W:
        raise ValueError(f"context parallel attention: heads ({H}, kv {Hk}) must be multiples of the group size {W}")
    if q.shape[0] % batch:
        raise ValueError("context parallel attention: token count must be a multiple of the batch")
    S = q.shape[0] // batch * W
    qh = _SeqToHead.apply(q, batch, W, group)
    kh = _SeqToHead.apply(k, batch, W, group)
    vh = _SeqToHead.apply(v, batch, W, group)
    krh = None
    if k_rope is not None:
        kr = k_rope.unsqueeze(1).expand(k_rope.shape[0], W, k_rope.shape[1])
        krh = _SeqToHead.apply(kr, batch, W, group).squeeze(1)
    out = attention(qh, kh, vh, krh, seq=S, causal=causal, window=window, scale=scale)
    return _HeadToSeq.apply(out, batch, W, group)


def shard_sequence(x: torch.Tensor, group=None) -> torch.Tensor:
    """[B, S, ...] -> this rank's chunk [B, S / W, ...]."""
    group = group if group is not None else dist.group.WORLD
    W, r = dist.get_world_size(group), dist.get_rank(group)
    if x.shape[1] % W:
        raise ValueError(f"sequence length {x.shape[1]} is not a multiple of the group size {W}")
    s = x.shape[1] // W
    return x[:, r * s:(r + 1) * s].contiguous()


def gather_sequence(x: torch.Tensor, group=None) -> torch.Tensor:
    """[B, s, ...] chunks of every rank -> [B, W * s, ...] (no gradient)."""
    group = group if group is not None else dist.group.WORLD
    W = dist.get_world_size(group)
    parts = [torch.empty_like(x) for _ in range(W)]
    dist.all_gather(parts, x.contiguous(), group=group)
    return torch.cat(parts, 1)


def positions(seq_len: int, group=None, device=None) -> torch.Tensor:
    """RoPE positions of this rank's chunk of a length-`seq_len` sequence."""
    group = group if group is not None else dist.group.WORLD
    W, r = dist.get_world_size(group), dist.get_rank(group)
    s = seq_len // W
    return torch.arange(r * s, (r + 1) * s, device=device)
