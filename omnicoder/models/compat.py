"""Compat model family: the reference's OmniTransformer architecture with its
module names (so its ``state_dict`` files load) and its observable behaviour.

Reference: src/omnicoder/modeling/transformer_moe.py:1016 (OmniTransformer),
:785 (Block), attention.py:349 (LatentKVAttention), moe_layer.py:36 (MoELayer),
routing.py, hrm.py, memory.py.  Behaviour kept on purpose (it is what a
reference checkpoint was trained with):
  * full-sequence passes are padded / truncated to compute_T = min(max_seq_len,
    128) positions and return logits for all compute_T positions
    (transformer_moe.py:1560-1585);
  * prefill attention: per head, the query latent (RoPE'd over interleaved pairs
    of the latent dim) attends over [8 landmark slots (zeros), M compressive
    slots, the last 16 rows of the padded K/V], where recent column c is hidden
    from query row r when c > r, scale 1/sqrt(latent dim)
    (attention.py:1135-1262);
  * decode keeps a 16-slot latent K/V shift register per layer and attends over
    all 16 slots; the query is rotated at position 0 (attention.py:1265-1612);
  * MoE: eval routes with the top-k router, sharpens the kept weights with an
    entropy-dependent temperature T = 0.8 + 0.4 * sigmoid(3 * H(last token's
    routing distribution)) (moe_layer.py:615-646), keeps at most `top_k`
    (token, k) pairs per expert (moe_scatter.py:548-554; pair p = token * k + j
    feeds and updates row p mod tokens, as the reference does) and runs
    fc1 -> GELU(tanh) -> fc2 experts with biases; training blends the top-k,
    multi-head and GRIN routers with softmax(_blend) weights and mixes shared
    experts in at 5 %;
  * each block scales its MoE output by sigmoid(5 * depth_gate_head(ln2(x)))
    (mixture-of-depths gate, transformer_moe.py:989-996);
  * HRM (3 planner/worker GRU rounds) runs after the blocks on full-sequence
    passes only.
Unlike the reference, routers and experts receive gradients here (the
reference detaches its expert banks, moe_layer.py:1056-1059).

All math is stock PyTorch: this family is for loading and running reference
checkpoints, not a benchmarked path.
"""
from __future__ import annotations

import math
from dataclasses import asdict, dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F

from .modules import (HRM, CompressiveKV, ExpertFFN, GRINGate, HierarchicalRouter, LandmarkIndexer,
                      MultiHeadRouter, RecurrentMemory, TopKRouter)


@dataclass
class CompatConfig:
    vocab_size: int = 32000
    n_layers: int = 4
    d_model: int = 512
    n_heads: int = 8
    mlp_dim: int = 2048
    n_experts: int = 4
    top_k: int = 2
    max_seq_len: int = 2048
    use_rope: bool = True
    kv_latent_dim: int = 256
    multi_query: bool = True
    multi_token: int = 1
    rope_scale: float = 1.0
    rope_base: float = 10000.0
    use_hrm: bool = True
    hrm_steps: int = 3
    hrm_adaptive: bool = False
    mem_slots: int = 0
    moe_group_sizes: list | None = None
    moe_sub_experts_per: int = 1
    moe_shared_general: int = 0
    compressive_slots: int = 0
    num_landmarks: int = 8
    decode_window: int = 16
    prefill_len: int = 128

    def to_dict(self):
        return asdict(self)


def _rope_tables(dim: int, n_pos: int, base: float, scale: float):
    inv = torch.exp(-torch.arange(0, dim, 2, dtype=torch.float64) / dim * math.log(base))
    t = torch.arange(n_pos, dtype=torch.float64) / (scale if scale != 0 else 1e-6)
    ang = torch.outer(t, inv)
    return ang.cos().float(), ang.sin().float()


def rope_interleaved(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate interleaved pairs (x0, x1) -> (x0 c - x1 s, x1 c + x0 s); x [..., T, D], cos/sin [T, D/2]."""
    x0, x1 = x[..., 0::2], x[..., 1::2]
    return torch.stack([x0 * cos - x1 * sin, x1 * cos + x0 * sin], -1).flatten(-2)


class LatentKVAttention(nn.Module):
    def __init__(self, c: CompatConfig):
        super().__init__()
        self.c = c
        D, H = c.d_model, c.n_heads
        self.n_heads, self.head_dim, self.dl = H, D // H, c.kv_latent_dim
        self.kv_out = self.head_dim if c.multi_query else D
        self.qkv_proj = nn.Linear(D, D + 2 * self.kv_out, bias=False)
        self.q_to_latent = nn.Linear(self.head_dim, self.dl, bias=False)
        self.k_to_latent = nn.Linear(self.head_dim, self.dl, bias=False)
        self.v_to_latent = nn.Linear(self.head_dim, self.dl, bias=False)
        self.kv_pair_to_latent = nn.Linear(self.head_dim, 2 * self.dl, bias=False)
        self.latent_is_head = self.dl == self.head_dim
        self.latent_to_head = None if self.latent_is_head else nn.Linear(self.dl, self.head_dim, bias=False)
        self.o_proj = nn.Linear(D, D, bias=False)
        self.landmarks = LandmarkIndexer(D, c.num_landmarks) if c.num_landmarks > 0 else None
        self.lm_to_head = nn.Linear(D, self.head_dim, bias=False) if c.num_landmarks > 0 else None
        self.compress_kv = CompressiveKV(self.dl, c.compressive_slots) if c.compressive_slots > 0 else None
        self.compute_T = min(c.max_seq_len, c.prefill_len)
        cos, sin = _rope_tables(self.dl, max(c.max_seq_len, self.compute_T), c.rope_base, c.rope_scale)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)

    def _latents(self, x):
        B, T, D = x.shape
        H, hd = self.n_heads, self.head_dim
        qkv = self.qkv_proj(x)
        q = qkv[..., :D].reshape(B, T, H, hd).transpose(1, 2)
        k_raw = qkv[..., D:D + self.kv_out]
        v_raw = qkv[..., D + self.kv_out:]
        q_lat = q if self.latent_is_head else self.q_to_latent(q)
        if self.c.multi_query:
            if self.latent_is_head:
                k_l, v_l = k_raw, v_raw
            else:
                kv = self.kv_pair_to_latent(k_raw)
                k_l, v_l = kv[..., :self.dl], kv[..., self.dl:]
            k_lat = k_l[:, None].expand(B, H, T, self.dl)
            v_lat = v_l[:, None].expand(B, H, T, self.dl)
        else:
            kh = k_raw.reshape(B, T, H, hd).transpose(1, 2)
            vh = v_raw.reshape(B, T, H, hd).transpose(1, 2)
            k_lat = kh if self.latent_is_head else self.k_to_latent(kh)
            v_lat = vh if self.latent_is_head else self.v_to_latent(vh)
        return q_lat, k_lat, v_lat

    def _out(self, y_lat):                     # [B, H, T, DL] -> [B, T, D]
        B, H, T, _ = y_lat.shape
        y = y_lat.transpose(1, 2)
        if self.latent_to_head is not None:
            y = self.latent_to_head(y)
        return self.o_proj(y.reshape(B, T, H * self.head_dim))

    def forward(self, x):
        """Full-sequence (prefill) pass; x is already padded to compute_T."""
        B, T, _ = x.shape
        q, k, v = self._latents(x)
        q = rope_interleaved(q, self.rope_cos[:T], self.rope_sin[:T])
        W = min(self.c.decode_window, T)
        Lk = self.c.num_landmarks
        M = self.c.compressive_slots
        parts_k = [k.new_zeros(B, self.n_heads, Lk, self.dl)]
        parts_v = [v.new_zeros(B, self.n_heads, Lk, self.dl)]
        if M > 0:
            km = k.new_zeros(B, self.n_heads, M, self.dl)
            vm = v.new_zeros(B, self.n_heads, M, self.dl)
            if self.compress_kv is not None:
                end = max(0, T - self.c.decode_window)
                ck, cv = self.compress_kv(k[:, :, :end], v[:, :, :end])
                km, vm = ck[:, :, :M], cv[:, :, :M]
            parts_k.append(km)
            parts_v.append(vm)
        parts_k.append(k[:, :, T - W:])
        parts_v.append(v[:, :, T - W:])
        kk = torch.cat(parts_k, 2)
        vv = torch.cat(parts_v, 2)
        s = torch.matmul(q, kk.transpose(-1, -2)) / math.sqrt(self.dl)
        rows = torch.arange(T, device=x.device)[:, None]
        cols = torch.arange(W, device=x.device)[None, :]
        mask = torch.zeros(T, kk.shape[2], device=x.device, dtype=s.dtype)
        mask[:, Lk + M:] = (cols > rows).to(s.dtype) * -1e9
        p = torch.softmax(s + mask, -1)
        return self._out(torch.matmul(p, vv)), k[:, :, T - W:], v[:, :, T - W:]

    def step(self, x, past_k, past_v):
        """One decode token x [B, 1, D] against the 16-slot shift register [B, H, W, DL]."""
        B = x.shape[0]
        q, k, v = self._latents(x)
        W = self.c.decode_window
        if past_k is None:
            past_k = k.new_zeros(B, self.n_heads, W, self.dl)
            past_v = v.new_zeros(B, self.n_heads, W, self.dl)
        nk = torch.cat([past_k[:, :, 1:], k], 2)
        nv = torch.cat([past_v[:, :, 1:], v], 2)
        q = rope_interleaved(q, self.rope_cos[:1], self.rope_sin[:1])   # position 0
        p = torch.softmax(torch.matmul(q, nk.transpose(-1, -2)) / math.sqrt(self.dl), -1)
        return self._out(torch.matmul(p, nv)), nk, nv


class MoELayer(nn.Module):
    def __init__(self, c: CompatConfig):
        super().__init__()
        D, E = c.d_model, c.n_experts
        self.n_experts, self.top_k = E, c.top_k
        self.num_shared_general = c.moe_shared_general
        if c.moe_group_sizes:
            self.router = HierarchicalRouter(D, E, group_sizes=c.moe_group_sizes, k=c.top_k)
            self._blend_enable = False
        else:
            self._router_topk = TopKRouter(D, E, k=c.top_k)
            self._router_multi = MultiHeadRouter(D, E, k=c.top_k, num_gates=4)
            self._router_grin = GRINGate(D, E, k=c.top_k)
            self._blend = nn.Parameter(torch.zeros(3))
            self._blend_enable = True
            self.router = self._router_topk
        self.experts = nn.ModuleList([ExpertFFN(D, c.mlp_dim) for _ in range(E)])
        self.shared = nn.ModuleList([ExpertFFN(D, c.mlp_dim) for _ in range(self.num_shared_general)]) \
            if self.num_shared_general > 0 else None
        self.vgr = (0.8, 1.2, 3.0)

    def forward(self, x):
        B, T, D = x.shape
        if self.training and self._blend_enable:
            ra, rb, rc = self._router_topk(x), self._router_multi(x), self._router_grin(x)
            w = torch.softmax(self._blend, 0)
            probs = w[0] * ra[2] + w[1] * rb[2] + w[2] * rc[2]
            vals, idx = torch.topk(probs, self.top_k, -1)
            scores = torch.softmax(vals, -1)
        else:
            idx, scores, probs, _ = self.router(x)
            if not self.training:
                tmin, tmax, lam = self.vgr
                p = probs[:, -1].clamp_min(1e-9)
                ent = -(p * p.log()).sum(-1).mean()
                temp = tmin + (tmax - tmin) * torch.sigmoid(lam * ent)
                scores = torch.softmax(scores / temp.clamp_min(1e-6), -1)
        scores = torch.nan_to_num(scores, nan=0.0, posinf=0.0, neginf=0.0)
        scores = scores / scores.sum(-1, keepdim=True).clamp_min(1e-8)
        xf = x.reshape(B * T, D)
        idx_f = idx.reshape(B * T, -1)
        sc_f = scores.reshape(B * T, -1)
        flat = idx_f.reshape(-1)
        # rank of each (token, k) pair inside its expert, in the order of the (unstable)
        # default sort of the flat expert ids -- the order the reference keeps pairs in
        # (moe_scatter.py:480-520); keep rank < top_k
        ids_sorted, order = torch.sort(flat)
        n = flat.numel()
        pos = torch.arange(n, device=flat.device)
        first = torch.ones(n, dtype=torch.bool, device=flat.device)
        first[1:] = ids_sorted[1:] != ids_sorted[:-1]
        start = torch.cummax(torch.where(first, pos, torch.zeros_like(pos)), 0).values
        rank = torch.empty_like(pos)
        rank[order] = pos - start
        keep = rank < self.expert_capacity(xf.shape[0])
        out = torch.zeros_like(xf)
        N = xf.shape[0]
        for e in range(self.n_experts):
            sel = ((flat == e) & keep).nonzero().squeeze(1)
            if sel.numel() == 0:
                continue
            # the reference maps flat pair p (= token * k + j) to row p mod N for both
            # the expert input and the combine target (moe_scatter.py:680-700, 828); kept
            # as is so that reference checkpoints reproduce their outputs
            tok = sel % N
            y = self.experts[e](xf[tok])
            out = out.index_add(0, tok, y * sc_f.reshape(-1)[sel, None])
        if self.training and self.shared is not None:
            share = sum(g(xf) for g in self.shared) / self.num_shared_general
            out = 0.95 * out + 0.05 * share
        return out.reshape(B, T, D)

    def expert_capacity(self, n_tokens: int) -> int:
        """Pairs kept per expert: top_k, the capacity the used layer passes to its dispatch
        (reference modeling/moe_layer.py)."""
        return self.top_k


class CapacityMoELayer(MoELayer):
    """The second MoE layer of the reference (modeling/transformer_moe.py:114-760, defined there
    but not used by the model): the same routers, experts and dispatch, with the per-expert
    capacity ceil(T * k / E * capacity_factor) (transformer_moe.py:615-621, `int(x + 0.9999)`),
    or `static_capacity` when given, instead of top_k."""

    def __init__(self, c: CompatConfig, capacity_factor: float = 1.2, static_capacity: int | None = None):
        super().__init__(c)
        self.capacity_factor = capacity_factor
        self.static_capacity = static_capacity

    def expert_capacity(self, n_tokens: int) -> int:
        if self.static_capacity is not None and self.static_capacity > 0:
            return int(self.static_capacity)
        expected = n_tokens * self.top_k / max(1, self.n_experts)
        return int(expected * self.capacity_factor + 0.9999)


class Block(nn.Module):
    def __init__(self, c: CompatConfig, layer: int):
        super().__init__()
        self.ln1 = nn.LayerNorm(c.d_model)
        self.attn = LatentKVAttention(c)
        self.ln2 = nn.LayerNorm(c.d_model)
        self.moe = MoELayer(c)
        self.depth_gate_head = nn.Linear(c.d_model, 1)
        self.mod_lambda = 5.0

    def _ffn(self, x):
        h = self.ln2(x)
        return x + self.moe(h) * torch.sigmoid(self.mod_lambda * self.depth_gate_head(h))

    def forward(self, x):
        a, k, v = self.attn(self.ln1(x))
        return self._ffn(x + a), k, v

    def step(self, x, pk, pv):
        a, k, v = self.attn.step(self.ln1(x), pk, pv)
        return self._ffn(x + a), k, v


class _LatentHead(nn.Module):
    """LayerNorm -> Linear -> GELU -> Linear (the reference's continuous latent and concept heads)."""

    def __init__(self, d_model: int, out_dim: int, attr: str, pooled_normalized: bool = False):
        super().__init__()
        self.attr, self.pooled_normalized = attr, pooled_normalized
        setattr(self, attr, nn.Sequential(nn.LayerNorm(d_model), nn.Linear(d_model, d_model), nn.GELU(),
                                          nn.Linear(d_model, out_dim)))

    def forward(self, h):
        if self.pooled_normalized:                       # concept head: last position, unit norm
            return F.normalize(getattr(self, self.attr)(h[:, -1] if h.dim() == 3 else h), dim=-1)
        return getattr(self, self.attr)(h)


class OmniTransformer(nn.Module):
    """Reference-compatible model.  Output contract (reference transformer_moe.py:1746-1809):
      use_cache=True  -> (logits, new_kv, mtp_logits, verifier_logits, diff, halt, retention)
      multi_token > 1 -> (logits, mtp_logits, diff, halt, retention)
      otherwise       -> (logits, None, None, image_latent, audio_latent, concept_latent, diff, halt,
                          retention)
    diff / halt / retention are sigmoid scores; `return_hidden=True` appends the
    final hidden states."""

    def __init__(self, **kw):
        super().__init__()
        c = CompatConfig(**{k: v for k, v in kw.items() if k in CompatConfig.__dataclass_fields__})
        self.c = c
        D, V = c.d_model, c.vocab_size
        self.vocab_size, self.d_model, self.multi_token = V, D, max(1, c.multi_token)
        self.embed = nn.Embedding(V, D)
        self.pos_embed = None if c.use_rope else nn.Parameter(torch.zeros(1, c.max_seq_len, D))
        self.blocks = nn.ModuleList([Block(c, i) for i in range(c.n_layers)])
        self.ln_f = nn.LayerNorm(D)
        self.lm_head = nn.Linear(D, V, bias=True)
        self.difficulty_head = nn.Linear(D, 1)
        self.halting_head = nn.Linear(D, 1)
        self.halting_critic = nn.Sequential(nn.LayerNorm(D), nn.Linear(D, D // 2), nn.GELU(), nn.Linear(D // 2, 1))
        self.verifier_head = nn.Linear(D, V, bias=False)
        self.retention_head = nn.Linear(D, 1)
        self.write_head = nn.Linear(D, 1)
        # continuous image / audio latent heads and the concept head (multimodal/aligner.py:54-97)
        self.image_latent_head = _LatentHead(D, 16, "proj")
        self.audio_latent_head = _LatentHead(D, 16, "proj")
        self.concept_head = _LatentHead(D, min(256, D), "net", pooled_normalized=True)
        self.hrm = HRM(D, steps=c.hrm_steps, adaptive_halting=c.hrm_adaptive) if c.use_hrm else None
        self.mtp_heads = nn.ModuleList([nn.Linear(D, V, bias=False) for _ in range(self.multi_token - 1)]) \
            if self.multi_token > 1 else None
        self.memory = RecurrentMemory(D, c.mem_slots) if c.mem_slots > 0 else None
        self.apply(self._init)

    @staticmethod
    def _init(m):
        if isinstance(m, (nn.Linear, nn.Embedding)):
            nn.init.normal_(m.weight, 0.0, 0.02)
            if getattr(m, "bias", None) is not None:
                nn.init.zeros_(m.bias)

    # ------------------------------------------------------------------
    def _heads(self, h):
        return (torch.sigmoid(self.difficulty_head(h)), torch.sigmoid(self.halting_head(h)),
                torch.sigmoid(self.retention_head(h)))

    def forward(self, input_ids, past_kv=None, use_cache: bool = False, return_hidden: bool = False):
        if use_cache:
            return self._decode(input_ids, past_kv, return_hidden)
        B, T = input_ids.shape
        cT = self.blocks[0].attn.compute_T if len(self.blocks) else T
        ids = input_ids[:, :cT]
        x = self.embed(ids)
        if x.shape[1] < cT:
            x = torch.cat([x, x.new_zeros(B, cT - x.shape[1], self.d_model)], 1)
        if self.pos_embed is not None:
            x = x + self.pos_embed[:, :cT]
        mem = self.memory(x) if self.memory is not None else None
        for blk in self.blocks:
            if mem is not None:
                x = blk(torch.cat([mem, x], 1))[0][:, mem.shape[1]:]
            else:
                x = blk(x)[0]
        if self.hrm is not None:
            x = self.hrm(x)
        h = self.ln_f(x)
        logits = self.lm_head(h)
        diff, halt, ret = self._heads(h)
        if self.mtp_heads is not None:
            out = (logits, [m(h) for m in self.mtp_heads], diff, halt, ret)
        else:
            out = (logits, None, None, self.image_latent_head(h), self.audio_latent_head(h), self.concept_head(h),
                   diff, halt, ret)
        return out + (h,) if return_hidden else out

    def _decode(self, input_ids, past_kv, return_hidden):
        x = self.embed(input_ids[:, -1:])
        if self.pos_embed is not None:
            x = x + self.pos_embed[:, :1]
        new_kv = []
        for i, blk in enumerate(self.blocks):
            pk, pv = (past_kv[i] if past_kv is not None else (None, None))
            x, k, v = blk.step(x, pk, pv)
            new_kv.append((k, v))
        h = self.ln_f(x)
        logits = self.lm_head(h)
        mtp = [m(h) for m in self.mtp_heads] if self.mtp_heads is not None else None
        diff, halt, ret = self._heads(h)
        out = (logits, new_kv, mtp, self.verifier_head(h), diff, halt, ret)
        return out + (h,) if return_hidden else out

    @torch.no_grad()
    def decode_next_id(self, input_ids, past_kv=None):
        """Greedy next token through the decode path; returns (ids [B, 1], new_kv)."""
        out = self.forward(input_ids, past_kv=past_kv, use_cache=True)
        return out[0][:, -1].argmax(-1, keepdim=True), out[1]


# ----------------------------------------------------------------------------
# reference state_dict loading
# ----------------------------------------------------------------------------
_PREFIXES = ("module.", "model.", "_orig_mod.", "net.")
_ALIAS_MARKERS = ("._attn_call._inner.", "._qkv_compiled.", "._qkv_call.", "._o_compiled.", "._o_call.",
                  "._query_to_latent_", "._kv_pair_to_latent_", "._key_to_latent_", "._value_to_latent_",
                  "._latent_to_head_", "._hrm_call.", "._work_w_cache", "._work_x_cache", "._prepacked_")


def normalize_reference_keys(sd: dict) -> dict:
    """Strip wrapper prefixes and `_orig_mod.` segments, drop aliases of other keys."""
    out = {}
    for k, v in sd.items():
        kk = k
        changed = True
        while changed:
            changed = False
            for p in _PREFIXES:
                if kk.startswith(p):
                    kk = kk[len(p):]
                    changed = True
        kk = kk.replace("._orig_mod.", ".")
        if any(m in "." + kk for m in _ALIAS_MARKERS):
            continue
        out[kk] = v
    return out


def load_reference_state_dict(model: OmniTransformer, sd: dict, strict: bool = False) -> dict:
    """Load a reference OmniTransformer checkpoint; returns a coverage report.
    Missing lm_head weights fall back to the tied embedding (the reference
    loader does the same, src/omnicoder/inference/generate.py:3558)."""
    for key in ("state_dict", "model", "module", "model_state_dict"):
        if isinstance(sd, dict) and key in sd and isinstance(sd[key], dict):
            sd = sd[key]
            break
    sd = normalize_reference_keys(sd)
    own = model.state_dict()
    usable = {k: v for k, v in sd.items() if k in own and tuple(v.shape) == tuple(own[k].shape)}
    if "lm_head.weight" not in usable and "embed.weight" in usable:
        usable["lm_head.weight"] = usable["embed.weight"]
    res = model.load_state_dict(usable, strict=False)
    report = {"loaded": len(usable), "model_keys": len(own), "checkpoint_keys": len(sd),
              "missing": sorted(res.missing_keys), "unexpected": sorted(k for k in sd if k not in own),
              "shape_mismatch": sorted(k for k, v in sd.items() if k in own and tuple(v.shape) != tuple(own[k].shape))}
    if strict and (report["missing"] or report["shape_mismatch"]):
        raise RuntimeError(f"incompatible checkpoint: {report}")
    return report
