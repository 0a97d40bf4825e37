"""Decoder-only LM of the spec family: RMSNorm, RoPE, MHA / GQA / MLA attention,
dense SwiGLU or routed-expert (+ shared expert) SwiGLU FFN, tied or untied
embeddings, optional multi-token-prediction and verifier heads.

What it replaces in the reference: OmniTransformer (src/omnicoder/modeling/
transformer_moe.py:1016) with LatentKVAttention (attention.py:349), MoELayer
(moe_layer.py:36) and the MTP/verifier heads (transformer_moe.py:1253-1399).
That model's quirks (128-token truncation, detached experts, 16-slot decode
window, LayerNorm/GELU experts) live in :mod:`omnicoder.models.compat`; this
family computes exact causal attention, routes with gradients and scales to
the long-context configs.

Layout notes (kernel-driven, converted by :meth:`OmniLM.export_state_dict`):
  * SwiGLU gate/up weights are one [2F, D] (or [E, 2F, D]) tensor with gate and
    up rows interleaved in blocks of 32 (the fused GEMM epilogue consumes pairs
    of 32-column accumulator chunks).
  * Residual adds are fused into the output-projection / down-projection GEMM
    epilogues: blocks take and return the residual stream.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from ..config import ModelConfig
from ..ops import (RopeTable, apply_rope, attention, attention_kv, embedding, layer_norm, linear, linear_rope,
                   lm_head_cross_entropy, moe_ffn, rms_norm, split_norm, swiglu_mlp)
from ..ops.decode import decode_attention
from ..ops.gemm import interleave_gate_up, split_gate_up


# device/dtype that parameters are created with (set by build_model)
_FACTORY: dict = {"device": "cpu", "dtype": torch.float32}


def _empty(*shape) -> torch.Tensor:
    return torch.empty(*shape, **_FACTORY)


def _ones(n: int) -> nn.Parameter:
    return nn.Parameter(torch.ones(n, **_FACTORY))


def _init(t: torch.Tensor, std: float) -> nn.Parameter:
    with torch.no_grad():
        t.normal_(0.0, std)
    return nn.Parameter(t)


class Norm(nn.Module):
    def __init__(self, dim: int, kind: str, eps: float):
        super().__init__()
        self.kind, self.eps = kind, eps
        self.weight = _ones(dim)
        self.bias = nn.Parameter(torch.zeros(dim, **_FACTORY)) if kind == "layernorm" else None

    def forward(self, x):
        if self.kind == "layernorm":
            return layer_norm(x, self.weight, self.bias, self.eps)
        return rms_norm(x, self.weight, self.eps)


def _tp_param(t: torch.Tensor) -> nn.Parameter:
    p = nn.Parameter(t.contiguous())
    p.tp_sharded = True
    return p


class GQAttention(nn.Module):
    """MHA (n_kv_heads == n_heads) or GQA with a fused QKV projection.  With a
    tensor-parallel context (`tp`, omnicoder.parallel.tensor) this rank holds
    n_heads / N query heads and n_kv_heads / N kv heads; the block input is its
    token shard (sequence parallel) and is all-gathered before the projection,
    the output projection's partial sums are reduce-scattered back."""

    def __init__(self, cfg: ModelConfig, tp=None):
        super().__init__()
        self.cfg = cfg
        self.tp = tp
        D, H, Hk, hd = cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        self.H, self.Hk, self.hd = H, Hk, hd
        self.wqkv = _init(_empty((H + 2 * Hk) * hd, D), cfg.init_std)
        self.wo = _init(_empty(D, H * hd), cfg.init_std)
        if tp is not None:
            h0, h1 = tp.shard(H, "query heads")
            k0, k1 = tp.shard(Hk, "kv heads")
            w = self.wqkv.data
            self.wqkv = _tp_param(torch.cat([w[h0 * hd:h1 * hd], w[(H + k0) * hd:(H + k1) * hd],
                                             w[(H + Hk + k0) * hd:(H + Hk + k1) * hd]]))
            self.wo = _tp_param(self.wo.data[:, h0 * hd:h1 * hd])
            self.H, self.Hk = h1 - h0, k1 - k0

    def qkv(self, y, rope: RopeTable, positions):
        T = y.shape[0]
        qkv = linear_rope(y, self.wqkv, rope, positions, self.hd, self.H + self.Hk,
                          interleaved=self.cfg.attn.rope_interleaved).view(T, self.H + 2 * self.Hk, self.hd)
        q = qkv[:, :self.H]
        k = qkv[:, self.H:self.H + self.Hk]
        v = qkv[:, self.H + self.Hk:]
        return q, k, v, None

    def forward(self, y, h, rope, positions, seq):
        if self.tp is not None and getattr(self.tp, "transport", "nccl") == "p2p":
            # fused collectives: the QKV GEMM gathers the token shards with its own loads, the output
            # projection's epilogue reduce-scatters its partial tiles (parallel/tensor.py)
            from ..parallel.tensor import tp_linear_ag, tp_linear_rs
            T = y.shape[0] * self.tp.world
            qkv = tp_linear_ag(y, self.wqkv, self.tp).view(T, self.H + 2 * self.Hk, self.hd)
            qkv = apply_rope(qkv, rope, positions, off=0, interleaved=self.cfg.attn.rope_interleaved,
                             heads=self.H + self.Hk)
            q, k, v = qkv[:, :self.H], qkv[:, self.H:self.H + self.Hk], qkv[:, self.H + self.Hk:]
            o = attention(q, k, v, None, seq=seq, causal=True, window=self.cfg.attn.window)
            return tp_linear_rs(o.reshape(T, -1), self.wo, self.tp, residual=h)
        if self.tp is not None and getattr(self.tp, "fp8", False):
            # block-scaled fp8 projections (fprop and dgrad), NCCL sequence-parallel collectives
            from ..ops.fp8 import fp8_linear
            from ..parallel.tensor import all_gather_seq, reduce_scatter_seq
            yf = all_gather_seq(y, self.tp)
            T = yf.shape[0]
            qkv = fp8_linear(yf, self.wqkv).view(T, self.H + 2 * self.Hk, self.hd)
            qkv = apply_rope(qkv, rope, positions, off=0, interleaved=self.cfg.attn.rope_interleaved,
                             heads=self.H + self.Hk)
            q, k, v = qkv[:, :self.H], qkv[:, self.H:self.H + self.Hk], qkv[:, self.H + self.Hk:]
            o = attention(q, k, v, None, seq=seq, causal=True, window=self.cfg.attn.window)
            return reduce_scatter_seq(fp8_linear(o.reshape(T, -1), self.wo), self.tp) + h
        if self.tp is not None:
            from ..parallel.tensor import all_gather_seq, reduce_scatter_seq
            yf = all_gather_seq(y, self.tp)
            q, k, v, kr = self.qkv(yf, rope, positions)
            o = attention(q, k, v, kr, seq=seq, causal=True, window=self.cfg.attn.window)
            return reduce_scatter_seq(linear(o.reshape(yf.shape[0], -1), self.wo), self.tp) + h
        q, k, v, kr = self.qkv(y, rope, positions)
        o = attention(q, k, v, kr, seq=seq, causal=True, window=self.cfg.attn.window)
        return linear(o.reshape(y.shape[0], -1), self.wo, residual=h)

    def forward_cached(self, y, h, rope, pos, cache, layer: int, prefill: bool):
        """New tokens y [B*Tn, D] at positions pos [B, Tn] against the cache."""
        B, Tn = pos.shape
        q, k, v, _ = self.qkv(y, rope, pos.reshape(-1))
        cache.write(layer, pos, k.reshape(B, Tn, self.Hk, self.hd), v.reshape(B, Tn, self.Hk, self.hd))
        if prefill and y.is_cuda and Tn % 128 == 0:
            o = attention(q, k, v, None, seq=Tn, causal=True, window=self.cfg.attn.window)
        else:
            kv_len = cache.lengths + Tn
            o = decode_attention(q.reshape(B, Tn, self.H, self.hd), cache.k[layer], cache.v[layer], pos, kv_len,
                                 window=self.cfg.attn.window, k_scale=cache.ks[layer], v_scale=cache.vs[layer],
                                 sink_rows=cache.sink, n_sink=cache.n_mem)
        return linear(o.reshape(B * Tn, -1), self.wo, residual=h)


class MLAttention(nn.Module):
    """Multi-head latent attention: keys/values come from a low-rank latent
    (kv_lora_rank) plus a shared rope key of qk_rope_dim."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        a = cfg.attn
        self.cfg = cfg
        D, H = cfg.d_model, cfg.n_heads
        self.H, self.dn, self.dr, self.dv, self.r = H, a.qk_nope_dim, a.qk_rope_dim, a.v_head_dim, a.kv_lora_rank
        self.wq = _init(_empty(H * (self.dn + self.dr), D), cfg.init_std)
        self.wkv_a = _init(_empty(self.r + self.dr, D), cfg.init_std)
        self.kv_norm = _ones(self.r)
        self.wkv_b = _init(_empty(H * (self.dn + self.dv), self.r), cfg.init_std)
        self.wo = _init(_empty(D, H * self.dv), cfg.init_std)

    def latent(self, y, rope: RopeTable, positions):
        """Compressed KV of the tokens: (normalised latent c [T, r], rotated rope key [T, dr])."""
        kva = linear_rope(y, self.wkv_a, rope, positions, self.r + self.dr, 1, off=self.r,
                          interleaved=self.cfg.attn.rope_interleaved)
        return split_norm(kva, self.kv_norm, self.r, self.cfg.norm_eps)

    def qkv_latent(self, y, rope: RopeTable, positions):
        """(q, k_nope view, v view, rope key, latent c) of tokens y."""
        T = y.shape[0]
        q = linear_rope(y, self.wq, rope, positions, self.dn + self.dr, self.H, off=self.dn,
                        interleaved=self.cfg.attn.rope_interleaved).view(T, self.H, self.dn + self.dr)
        c, kr = self.latent(y, rope, positions)
        kv = linear(c, self.wkv_b).view(T, self.H, self.dn + self.dv)
        return q, kv[:, :, :self.dn], kv[:, :, self.dn:], kr, c

    def qkv(self, y, rope: RopeTable, positions):
        return self.qkv_latent(y, rope, positions)[:4]

    def forward(self, y, h, rope, positions, seq):
        T = y.shape[0]
        q = linear_rope(y, self.wq, rope, positions, self.dn + self.dr, self.H, off=self.dn,
                        interleaved=self.cfg.attn.rope_interleaved).view(T, self.H, self.dn + self.dr)
        c, kr = self.latent(y, rope, positions)
        kv = linear(c, self.wkv_b).view(T, self.H, self.dn + self.dv)
        o = attention_kv(q, kv, self.dn, kr, seq=seq, causal=True, window=self.cfg.attn.window,
                         scale=1.0 / math.sqrt(self.dn + self.dr))
        return linear(o.reshape(T, -1), self.wo, residual=h)

    @torch.no_grad()
    def prepare_inference(self):
        """Absorb the latent up-projections into the query and output projections:
        q_lat[h] = W_uk[h]^T q_nope[h] and out = sum_h Wo_h W_uv[h] o_lat[h], so decoding
        attends over the compressed latent cache directly."""
        H, dn, dr, dv, r = self.H, self.dn, self.dr, self.dv, self.r
        D = self.wq.shape[1]
        wkv_b = self.wkv_b.float().view(H, dn + dv, r)
        w_uk, w_uv = wkv_b[:, :dn], wkv_b[:, dn:]
        wq = self.wq.float().view(H, dn + dr, D)
        wq_lat = torch.einsum("hnr,hnd->hrd", w_uk, wq[:, :dn])
        self.wq_abs = torch.cat([wq_lat, wq[:, dn:]], dim=1).reshape(H * (r + dr), D).to(self.wq.dtype).contiguous()
        wo = self.wo.float().view(D, H, dv)
        self.wo_abs = torch.einsum("dhv,hvr->dhr", wo, w_uv).reshape(D, H * r).to(self.wo.dtype).contiguous()

    def forward_cached(self, y, h, rope, pos, cache, layer: int, prefill: bool):
        B, Tn = pos.shape
        flat = pos.reshape(-1)
        if prefill and y.is_cuda and Tn % 128 == 0:
            q, k, v, kr, c = self.qkv_latent(y, rope, flat)
            cache.write(layer, pos, torch.cat([c, kr], dim=-1).view(B, Tn, -1))
            o = attention(q, k, v, kr, seq=Tn, causal=True, window=self.cfg.attn.window,
                          scale=1.0 / math.sqrt(self.dn + self.dr))
            return linear(o.reshape(B * Tn, -1), self.wo, residual=h)
        if getattr(self, "wq_abs", None) is None:
            self.prepare_inference()
        r, dr = self.r, self.dr
        qa = linear_rope(y, self.wq_abs, rope, flat, r + dr, self.H, off=r,
                         interleaved=self.cfg.attn.rope_interleaved).view(B, Tn, self.H, r + dr)
        c, kr = self.latent(y, rope, flat)
        cache.write(layer, pos, torch.cat([c, kr], dim=-1).view(B, Tn, r + dr))
        kv_len = cache.lengths + Tn
        o = decode_attention(qa, cache.k[layer], None, pos, kv_len, window=self.cfg.attn.window,
                             scale=1.0 / math.sqrt(self.dn + self.dr), k_scale=cache.ks[layer], latent_v_dim=r,
                             sink_rows=cache.sink, n_sink=cache.n_mem)
        return linear(o.reshape(B * Tn, -1), self.wo_abs, residual=h)


class DenseFFN(nn.Module):
    """SwiGLU MLP.  With `tp` this rank holds F / N hidden features (a contiguous
    slice of the 32-row interleaved gate/up rows) and runs sequence parallel."""

    def __init__(self, D: int, F: int, std: float, tp=None):
        super().__init__()
        self.tp = tp
        self.w13 = _init(_empty(2 * F, D), std)
        self.w2 = _init(_empty(D, F), std)
        if tp is not None:
            f0, f1 = tp.shard(F, "ffn dim")
            if (f1 - f0) % 32:
                raise ValueError("tensor-parallel ffn shards must be multiples of 32 features")
            self.w13 = _tp_param(self.w13.data[2 * f0:2 * f1])
            self.w2 = _tp_param(self.w2.data[:, f0:f1])

    def forward(self, y, h):
        if self.tp is not None and getattr(self.tp, "transport", "nccl") == "p2p":
            from ..parallel.tensor import tp_swiglu_mlp
            return tp_swiglu_mlp(y, self.w13, self.w2, self.tp, residual=h), None
        if self.tp is not None:
            from ..parallel.tensor import all_gather_seq, reduce_scatter_seq
            if getattr(self.tp, "fp8", False):
                from ..ops.fp8 import fp8_swiglu_mlp
                return reduce_scatter_seq(fp8_swiglu_mlp(all_gather_seq(y, self.tp), self.w13, self.w2),
                                          self.tp) + h, None
            return reduce_scatter_seq(swiglu_mlp(all_gather_seq(y, self.tp), self.w13, self.w2), self.tp) + h, None
        return swiglu_mlp(y, self.w13, self.w2, residual=h), None


class MoEFFN(nn.Module):
    """Routed SwiGLU experts (+ shared experts).  With an expert-parallel layout
    (`ep`, see omnicoder.parallel.expert_data) this rank holds experts
    [lo, hi) of the group; the full stack is still drawn from the RNG so that
    every layout initialises identically to the single-device model."""

    def __init__(self, cfg: ModelConfig, ep=None):
        super().__init__()
        m = cfg.moe
        D = cfg.d_model
        self.cfg = cfg
        self.ep = ep
        self.router = _init(_empty(m.n_experts, D), cfg.init_std)
        lo, hi = ep.expert_slice(m.n_experts) if ep is not None else (0, m.n_experts)
        self.w13 = _init(_empty(m.n_experts, 2 * m.ffn_dim, D), cfg.init_std)
        self.w2 = _init(_empty(m.n_experts, D, m.ffn_dim), cfg.init_std)
        if ep is not None:
            self.w13 = nn.Parameter(self.w13.data[lo:hi].clone())
            self.w2 = nn.Parameter(self.w2.data[lo:hi].clone())
        self.shared = DenseFFN(D, m.ffn_dim * m.n_shared_experts, cfg.init_std) if m.n_shared_experts > 0 else None
        self.aux_grad_scale = 1.0
        self.top_k_override: int | None = None   # decode-time adaptive expert count (inference add-on)

    def forward(self, y, h):
        m = self.cfg.moe
        k = self.top_k_override or m.top_k
        T = y.shape[0]
        base = self.shared(y, h)[0] if self.shared is not None else h
        if self.ep is not None:
            from ..parallel.expert import ep_moe_ffn
            world = self.ep.world
            out, aux = ep_moe_ffn(y, self.router, self.w13, self.w2, k, self.ep.ep, m.capacity(T * world),
                                  m.renorm_topk, m.aux_loss_alpha, m.z_loss_beta, add=base,
                                  aux_grad_scale=self.aux_grad_scale)
            return out, aux
        out, aux = moe_ffn(y, self.router, self.w13, self.w2, k, m.capacity(T), m.renorm_topk,
                           m.aux_loss_alpha, m.z_loss_beta, add=base, aux_grad_scale=self.aux_grad_scale)
        return out, aux


class Block(nn.Module):
    def __init__(self, cfg: ModelConfig, layer: int, ep=None, tp=None):
        super().__init__()
        if tp is not None and (cfg.attn.kind == "mla" or cfg.is_moe_layer(layer)):
            raise NotImplementedError("tensor parallelism covers dense GQA/MHA blocks; use expert parallelism for MoE")
        self.attn_norm = Norm(cfg.d_model, cfg.norm, cfg.norm_eps)
        self.attn = MLAttention(cfg) if cfg.attn.kind == "mla" else GQAttention(cfg, tp)
        self.ffn_norm = Norm(cfg.d_model, cfg.norm, cfg.norm_eps)
        self.ffn = MoEFFN(cfg, ep) if cfg.is_moe_layer(layer) else DenseFFN(cfg.d_model, cfg.ffn_dim, cfg.init_std, tp)

    def forward(self, h, rope, positions, seq):
        h = self.attn(self.attn_norm(h), h, rope, positions, seq)
        return self.ffn(self.ffn_norm(h), h)

    def forward_cached(self, h, rope, pos, cache, layer: int, prefill: bool):
        h = self.attn.forward_cached(self.attn_norm(h), h, rope, pos, cache, layer, prefill)
        return self.ffn(self.ffn_norm(h), h)[0]


class OmniLM(nn.Module):
    """The spec-family language model.  `forward(ids, labels)` returns a dict with
    `loss` (CE + auxiliary), `ce`, `aux` and, without labels, `logits` of the last
    position (or all positions with `all_logits=True`)."""

    def __init__(self, cfg: ModelConfig, ep=None, tp=None):
        super().__init__()
        self.cfg = cfg
        self.tp = tp
        D, V = cfg.d_model, cfg.vocab_size
        self.embed = _init(_empty(V, D), cfg.init_std)
        self.blocks = nn.ModuleList([Block(cfg, i, ep, tp) for i in range(cfg.n_layers)])
        self.norm_f = Norm(D, cfg.norm, cfg.norm_eps)
        self.lm_head = None if cfg.tie_embeddings else _init(_empty(V, D), cfg.init_std)
        self.mtp_heads = nn.ParameterList([_init(_empty(V, D), cfg.init_std) for _ in range(cfg.mtp_heads)])
        self.verifier = _init(_empty(V, D), cfg.init_std) if cfg.verifier_head else None
        rot = cfg.attn.qk_rope_dim if cfg.attn.kind == "mla" else cfg.head_dim
        self.rope = RopeTable(rot, cfg.max_seq_len, cfg.attn.rope_theta, cfg.attn.rope_scale)

    # ------------------------------------------------------------------
    @property
    def head_weight(self) -> torch.Tensor:
        return self.embed if self.lm_head is None else self.lm_head

    def set_aux_grad_scale(self, s: float):
        for b in self.blocks:
            if isinstance(b.ffn, MoEFFN):
                b.ffn.aux_grad_scale = s

    def hidden(self, ids: torch.Tensor | None, positions: torch.Tensor | None = None,
               embeds: torch.Tensor | None = None):
        """Final normalised hidden states [B*S, D] and the summed auxiliary loss.  `embeds`
        [B, S, D] replaces the token embeddings (inputs composed with other modalities)."""
        B, S = (embeds.shape[:2] if embeds is not None else ids.shape)
        dev = embeds.device if embeds is not None else ids.device
        if dev.type == "cuda":
            self.rope.to(dev)
        if embeds is not None:
            if self.tp is not None:
                raise NotImplementedError("input embeddings with tensor parallelism")
            h = embeds.reshape(B * S, -1).to(self.embed.dtype).contiguous()
        else:
            flat = ids.reshape(-1)
            if self.tp is not None:                       # sequence parallel: this rank's token shard
                from ..parallel.tensor import scatter_seq
                flat = scatter_seq(flat, self.tp)
            h = embedding(flat, self.embed)
        if positions is None:
            positions = torch.arange(S, device=dev).repeat(B)
        aux_total = None
        for blk in self.blocks:
            h, aux = blk(h, self.rope, positions, S)
            if aux is not None:
                aux_total = aux if aux_total is None else aux_total + aux
        return self.norm_f(h), aux_total

    def forward(self, ids: torch.Tensor | None, labels: torch.Tensor | None = None, all_logits: bool = False,
                assume_all_valid: bool = False, embeds: torch.Tensor | None = None):
        y, aux = self.hidden(ids, embeds=embeds)
        if ids is None:
            ids = torch.empty(embeds.shape[:2], dtype=torch.long, device=embeds.device)   # shape carrier
        out = {}
        if labels is not None and self.tp is not None:
            from ..parallel.tensor import scatter_seq
            labels = scatter_seq(labels.reshape(-1), self.tp)
        if labels is not None:
            ce = lm_head_cross_entropy(y, self.head_weight, labels, assume_all_valid=assume_all_valid)
            loss = ce
            if self.cfg.mtp_heads > 0:
                B, S = ids.shape
                for j, w in enumerate(self.mtp_heads):
                    shift = j + 1
                    lab = torch.full_like(labels, -100)
                    lab[:, :S - shift] = labels[:, shift:]
                    loss = loss + 0.5 * lm_head_cross_entropy(y, w, lab)
            out["ce"] = ce
            out["aux"] = aux if aux is not None else torch.zeros((), device=ids.device)
            out["loss"] = loss + (aux if aux is not None else 0.0)
        else:
            B, S = ids.shape
            yy = y if all_logits else y.view(B, S, -1)[:, -1]
            out["logits"] = linear(yy, self.head_weight).float().view(B, S if all_logits else 1, -1)
        return out

    # ------------------------------------------------------------------
    @torch.no_grad()
    def forward_cached(self, ids: torch.Tensor, cache, prefill: bool = False, last_only: bool = False,
                       return_hidden: bool = False, embeds: torch.Tensor | None = None):
        """Process new tokens ids [B, Tn] against `cache` (appending them) and return
        logits [B, Tn, V] (or [B, 1, V] with last_only).  `prefill=True` asserts the
        cache is empty, which lets long prompts use the flash-attention kernels.
        `return_hidden`: also return the final normalised hidden states of the same
        positions ([B, Tn or 1, D]).  `embeds` [B, Tn, D]: input vectors used in place of
        the token embeddings (priming the cache with features, e.g. another modality's)."""
        B, Tn = ids.shape
        if ids.is_cuda:
            self.rope.to(ids.device)
        pos = cache.positions(Tn)
        if embeds is not None:
            h = embeds.reshape(B * Tn, -1).to(self.embed.dtype).contiguous()
        else:
            h = embedding(ids.reshape(-1), self.embed)
        for i, blk in enumerate(self.blocks):
            h = blk.forward_cached(h, self.rope, pos, cache, i, prefill)
        cache.advance(Tn)
        y = self.norm_f(h).view(B, Tn, -1)
        if last_only:
            y = y[:, -1:]
        logits = linear(y.reshape(-1, y.shape[-1]), self.head_weight).float().view(B, y.shape[1], -1)
        return (logits, y) if return_hidden else logits

    def prepare_inference(self):
        for b in self.blocks:
            if isinstance(b.attn, MLAttention):
                b.attn.prepare_inference()
        return self

    def export_state_dict(self) -> dict[str, torch.Tensor]:
        """state_dict with SwiGLU gate/up split into separate `w1`/`w3` tensors."""
        sd = {}
        for k, v in self.state_dict().items():
            if k.endswith(".w13"):
                w1, w3 = split_gate_up(v)
                sd[k[:-4] + ".w1"] = w1
                sd[k[:-4] + ".w3"] = w3
            else:
                sd[k] = v
        return sd

    def load_export_state_dict(self, sd: dict[str, torch.Tensor], strict: bool = True):
        merged = {}
        for k, v in sd.items():
            if k.endswith(".w1"):
                merged[k[:-3] + ".w13"] = interleave_gate_up(v, sd[k[:-3] + ".w3"])
            elif k.endswith(".w3"):
                continue
            else:
                merged[k] = v
        return self.load_state_dict(merged, strict=strict)


def build_model(cfg: ModelConfig, device="cpu", dtype=None, seed: int | None = 0, ep=None, tp=None) -> OmniLM:
    """Random-init model N(0, init_std) created directly on `device` (bf16 on CUDA,
    fp32 on CPU by default).  `ep`: an expert-parallel layout
    (omnicoder.parallel.expert_data.ExpertDataParallel) -- the model then holds
    only this rank's routed experts."""
    global _FACTORY
    if seed is not None:
        torch.manual_seed(seed)
        if str(device).startswith("cuda"):
            torch.cuda.manual_seed(seed)
    if dtype is None:
        dtype = torch.bfloat16 if str(device).startswith("cuda") else torch.float32
    old = _FACTORY
    _FACTORY = {"device": torch.device(device), "dtype": dtype}
    try:
        m = OmniLM(cfg, ep, getattr(tp, "tp", tp))
    finally:
        _FACTORY = old
    m.rope.to(device)
    return m
