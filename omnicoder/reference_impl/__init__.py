"""fp32 CPU oracle of the spec model family, written independently of
:mod:`omnicoder.models` so the two can check each other.

Plain PyTorch, no fused ops, no custom autograd: RMSNorm, half-split RoPE,
multi-head causal attention, a softmax top-k router with renormalisation over
SwiGLU experts (dropless), tied embeddings, AdamW (torch.optim), and greedy
decoding with a per-layer key/value cache.

Weights are taken from an :class:`omnicoder.models.lm.OmniLM` state_dict (MHA
attention, dense or MoE FFN) so that both implementations run the same
parameters.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def rms_norm(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def rope_angles(positions, rot, theta, scale):
    inv = 1.0 / (theta ** (torch.arange(0, rot, 2, dtype=torch.float64) / rot))
    ang = (positions.double()[:, None] / scale) * inv[None, :]
    return ang.cos().float(), ang.sin().float()


def rope_half(x, cos, sin):
    # x [..., T, D]; cos/sin [T, D/2]
    h = x.shape[-1] // 2
    a, b = x[..., :h], x[..., h:]
    return torch.cat([a * cos - b * sin, b * cos + a * sin], dim=-1)


def split_w13(w13, block=32):
    """Separate interleaved gate/up rows (blocks of 32) into (w1, w3)."""
    F2 = w13.shape[-2]
    v = w13.reshape(*w13.shape[:-2], F2 // (2 * block), 2, block, w13.shape[-1])
    return (v[..., 0, :, :].reshape(*w13.shape[:-2], F2 // 2, w13.shape[-1]),
            v[..., 1, :, :].reshape(*w13.shape[:-2], F2 // 2, w13.shape[-1]))


class ReferenceLM(torch.nn.Module):
    def __init__(self, cfg, state_dict):
        super().__init__()
        assert cfg.attn.kind == "mha", "the oracle covers multi-head attention"
        self.cfg = cfg
        self.p = torch.nn.ParameterDict()
        for k, v in state_dict.items():
            self.p[k.replace(".", "__")] = torch.nn.Parameter(v.detach().clone().float())

    def w(self, name):
        return self.p[name.replace(".", "__")]

    # ------------------------------------------------------------------
    def _ffn(self, i, x):
        c = self.cfg
        if c.is_moe_layer(i):
            m = c.moe
            logits = x @ self.w(f"blocks.{i}.ffn.router").t()
            probs = torch.softmax(logits, -1)
            topw, topi = probs.topk(m.top_k, dim=-1)
            if m.renorm_topk:
                topw = topw / topw.sum(-1, keepdim=True)
            out = torch.zeros_like(x)
            w1, w3 = split_w13(self.w(f"blocks.{i}.ffn.w13"))
            w2 = self.w(f"blocks.{i}.ffn.w2")
            for e in range(m.n_experts):
                y = (F.silu(x @ w1[e].t()) * (x @ w3[e].t())) @ w2[e].t()
                gate = (topw * (topi == e)).sum(-1, keepdim=True)
                out = out + gate * y
            if m.n_shared_experts:
                s1, s3 = split_w13(self.w(f"blocks.{i}.ffn.shared.w13"))
                out = out + (F.silu(x @ s1.t()) * (x @ s3.t())) @ self.w(f"blocks.{i}.ffn.shared.w2").t()
            return out
        w1, w3 = split_w13(self.w(f"blocks.{i}.ffn.w13"))
        return (F.silu(x @ w1.t()) * (x @ w3.t())) @ self.w(f"blocks.{i}.ffn.w2").t()

    def _attn(self, i, x, positions, cache):
        c = self.cfg
        B, T, D = x.shape
        H, hd = c.n_heads, c.head_dim
        qkv = x @ self.w(f"blocks.{i}.attn.wqkv").t()
        q, k, v = qkv.view(B, T, 3, H, hd).unbind(2)
        cos, sin = rope_angles(positions, hd, c.attn.rope_theta, c.attn.rope_scale)
        q = rope_half(q.transpose(1, 2), cos, sin)
        k = rope_half(k.transpose(1, 2), cos, sin)
        v = v.transpose(1, 2)
        if cache is not None:
            if i in cache:
                k = torch.cat([cache[i][0], k], dim=2)
                v = torch.cat([cache[i][1], v], dim=2)
            cache[i] = (k, v)
        S = k.shape[2]
        s = (q @ k.transpose(-1, -2)) / math.sqrt(hd)
        qpos = positions[:, None]
        kpos = torch.arange(S)[None, :]
        s = s.masked_fill(kpos > qpos, float("-inf"))
        o = torch.softmax(s, -1) @ v
        return o.transpose(1, 2).reshape(B, T, H * hd) @ self.w(f"blocks.{i}.attn.wo").t()

    def forward(self, ids, positions=None, cache=None):
        c = self.cfg
        B, T = ids.shape
        if positions is None:
            positions = torch.arange(T)
        h = self.w("embed")[ids]
        for i in range(c.n_layers):
            h = h + self._attn(i, rms_norm(h, self.w(f"blocks.{i}.attn_norm.weight"), c.norm_eps), positions, cache)
            h = h + self._ffn(i, rms_norm(h, self.w(f"blocks.{i}.ffn_norm.weight"), c.norm_eps))
        h = rms_norm(h, self.w("norm_f.weight"), c.norm_eps)
        head = self.w("embed") if c.tie_embeddings else self.w("lm_head")
        return h @ head.t()

    def loss(self, ids, labels):
        logits = self.forward(ids)
        return F.cross_entropy(logits.reshape(-1, logits.shape[-1]), labels.reshape(-1))

    @torch.no_grad()
    def greedy(self, prompt, n_new):
        cache = {}
        T = prompt.shape[1]
        logits = self.forward(prompt, torch.arange(T), cache)
        out = []
        nxt = logits[:, -1].argmax(-1)
        for step in range(n_new):
            out.append(nxt)
            pos = torch.tensor([T + step])
            logits = self.forward(nxt[:, None], pos, cache)
            nxt = logits[:, -1].argmax(-1)
        return torch.stack(out, dim=1)
