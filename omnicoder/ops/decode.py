"""Attention of new query tokens against a key/value cache (decode and
speculative verification).

    q       [B, Tn, H, Dq]     new queries (already rotated)
    cache   per-layer tensors of omnicoder.inference.kv_cache.KVCache
    q_pos   [B, Tn]            absolute positions of the queries
Keys visible to query (b, t): positions p < lengths_after[b] with p <= q_pos[b, t]
and, with a window, p > q_pos[b, t] - window.

MHA/GQA: keys/values [B, L, Hk, D].  MLA (absorbed): the latent cache
[B, L, r + dr] is both the key (all r + dr dims, against q = [q_latent, q_rope])
and the value (first r dims); the output is the latent o [B, Tn, H, r] that the
absorbed output projection consumes.

CUDA: MLA latent caches of the model sizes (576/512, 320/256) run a tcgen05
kernel (keys on the MMA M side, query rows on N, any number of query rows);
other layouts run the split-KV CUDA-core kernel (<= 64 query rows per call).
Both take bf16 or int8 (per-token / per-head scaled) caches.  CPU: dense
masked softmax (the oracle).
"""
from __future__ import annotations

import math

import torch

from . import _ext


def decode_attention_torch(q, k, v, q_pos, kv_len, *, window=0, scale=None, k_scale=None, v_scale=None,
                           latent_v_dim=0, sink_rows=0, n_sink=0):
    """k: [B, L, Hk, D] (or latent [B, L, D] when latent_v_dim > 0); scales dequantise int8 caches.
    Token position p is cache row sink_rows + p; rows [0, n_sink) are memory every query sees."""
    B, Tn, H, Dq = q.shape
    sc = scale if scale is not None else 1.0 / math.sqrt(Dq)
    if latent_v_dim:
        kf = k.float() if k_scale is None else k.float() * k_scale.float()[..., None]
        kf = kf[:, :, None, :]                         # [B, L, 1, D]
        vf = kf[..., :latent_v_dim]
    else:
        kf = k.float() if k_scale is None else k.float() * k_scale.float()[..., None]
        vf = v.float() if v_scale is None else v.float() * v_scale.float()[..., None]
    L, Hk = kf.shape[1], kf.shape[2]
    rep = H // Hk
    kk = kf.permute(0, 2, 1, 3).repeat_interleave(rep, dim=1)   # [B, H, L, D]
    vv = vf.permute(0, 2, 1, 3).repeat_interleave(rep, dim=1)
    qq = q.float().permute(0, 2, 1, 3)                           # [B, H, Tn, D]
    s = torch.matmul(qq, kk.transpose(-1, -2)) * sc              # [B, H, Tn, L]
    rows = torch.arange(L, device=q.device)
    p = rows - sink_rows
    qp = q_pos[:, None, :, None]
    mask = (p[None, None, None, :] > qp) | (p[None, None, None, :] >= kv_len[:, None, None, None]) | \
        (p[None, None, None, :] < 0)
    if window > 0:
        mask |= p[None, None, None, :] <= qp - window
    if n_sink > 0:
        mask &= ~(rows < n_sink)[None, None, None, :]
    s = s.masked_fill(mask, float("-inf"))
    o = torch.matmul(torch.softmax(s, -1), vv)                   # [B, H, Tn, Dv]
    return o.permute(0, 2, 1, 3).to(q.dtype)


def decode_attention(q, k, v, q_pos, kv_len, *, window=0, scale=None, k_scale=None, v_scale=None,
                     latent_v_dim=0, sink_rows=0, n_sink=0):
    if not q.is_cuda:
        return decode_attention_torch(q, k, v, q_pos, kv_len, window=window, scale=scale, k_scale=k_scale,
                                      v_scale=v_scale, latent_v_dim=latent_v_dim, sink_rows=sink_rows,
                                      n_sink=n_sink)
    C = _ext.load()
    sc = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    B, Tn, H, _ = q.shape
    Hk = 1 if latent_v_dim else k.shape[2]
    G = H // Hk
    step = max(1, C.decode_rows_limit(q.shape[-1], latent_v_dim or (v.shape[-1] if v is not None else 0),
                                      bool(latent_v_dim), Hk) // G)   # query rows one call takes
    qp = q_pos.to(torch.int32)
    kl = kv_len.to(torch.int32).contiguous()
    if Tn <= step:
        return C.attn_decode(q.contiguous(), k, v, k_scale, v_scale, qp.contiguous(), kl, window, sc, latent_v_dim,
                             sink_rows, n_sink)
    outs = [C.attn_decode(q[:, t:t + step].contiguous(), k, v, k_scale, v_scale, qp[:, t:t + step].contiguous(), kl,
                          window, sc, latent_v_dim, sink_rows, n_sink) for t in range(0, Tn, step)]
    return torch.cat(outs, dim=1)
