"""Model building blocks of the reference architecture, as plain PyTorch modules.

Everything here runs on any device with stock torch ops; the compat model
family (:mod:`omnicoder.models.compat`) and optional features of the spec
family use them.  None of these is on the benchmarked hot path.

Routers (reference src/omnicoder/modeling/routing.py): every router maps
x [B, T, C] to (idx [B, T, k], scores [B, T, k], probs_full [B, T, E], aux)
where `scores` are the combine weights of the selected experts and `aux` holds
load statistics (importance = mean routing probability, load = share of the
k * B * T assignments, z_loss = mean logsumexp^2).
  TopKRouter            linear gate (+ conditioning bias), training-time
                        jitter / Gumbel noise / expert dropout, temperature,
                        top-k on logits, softmax over the kept logits.
  HierarchicalRouter    group gate picks one contiguous expert group per token
                        (argmax), experts outside it are masked.
  MultiHeadRouter       mean of G softmax gates, renormalised top-k.
  GRINGate              logits scaled by 1 / (1 + difficulty), straight-through
                        one-hot selection.
  LLMRouter             one causal self-attention + FF layer of context before
                        the gate.
  InteractionRouter     gate over [x, projected condition].
Other blocks: HRM (planner/worker GRUs, hrm.py), RecurrentMemory,
CompressiveKV, LandmarkIndexer (memory.py), GatedMambaSSM / GatedConvSSM
(ssm.py), HyenaMixer1D (hyena.py), ExpertFFN (experts.py).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F


def _aux_stats(probs: torch.Tensor, idx: torch.Tensor, logits: torch.Tensor | None, E: int) -> dict:
    with torch.no_grad():
        importance = probs.reshape(-1, E).mean(0)
        counts = torch.bincount(idx.reshape(-1), minlength=E).to(probs.dtype)
        load = counts / counts.sum().clamp_min(1.0)
    aux = {"importance": importance, "load": load}
    if logits is not None:
        z = torch.logsumexp(logits, dim=-1)
        aux["z_loss"] = (z * z).mean()
    return aux


def _gumbel(t: torch.Tensor, eps: float = 1e-9) -> torch.Tensor:
    u = torch.rand_like(t)
    return -torch.log(-torch.log(u + eps) + eps)


class TopKRouter(nn.Module):
    def __init__(self, d_model: int, n_experts: int, k: int = 2, temperature: float = 1.0, jitter_noise: float = 0.0,
                 use_gumbel: bool = False, expert_dropout_p: float = 0.0):
        super().__init__()
        self.n_experts, self.k = n_experts, k
        self.temperature = max(1e-6, float(temperature))
        self.jitter_noise, self.use_gumbel = float(jitter_noise), bool(use_gumbel)
        self.expert_dropout_p = min(1.0, max(0.0, float(expert_dropout_p)))
        self.gate = nn.Linear(d_model, n_experts, bias=False)
        self.cond_proj = nn.Linear(d_model, n_experts, bias=False)
        self.sample_gumbel_topk = False

    def forward(self, x: torch.Tensor, cond: dict | None = None):
        logits = self.gate(x)
        if cond:
            for key in ("image", "text", "audio", "video"):
                c = cond.get(key)
                if isinstance(c, torch.Tensor):
                    logits = logits + self.cond_proj(c).unsqueeze(1)
                    break
        if self.training and self.jitter_noise > 0:
            noise = _gumbel(logits) if self.use_gumbel else torch.randn_like(logits)
            logits = logits + self.jitter_noise * noise
        if self.training and self.expert_dropout_p > 0:
            drop = torch.rand_like(logits) < self.expert_dropout_p
            keep_best = F.one_hot(logits.argmax(-1), self.n_experts).bool()
            logits = logits.masked_fill(drop & ~keep_best, torch.finfo(logits.dtype).min)
        logits = logits / self.temperature
        probs = torch.softmax(logits, -1)
        sel = logits + _gumbel(logits) if (self.training and self.sample_gumbel_topk) else logits
        vals, idx = torch.topk(sel, self.k, dim=-1)
        if sel is not logits:
            vals = logits.gather(-1, idx)
        scores = torch.softmax(vals, -1)
        return idx, scores, probs, _aux_stats(probs, idx, logits, self.n_experts)


class HierarchicalRouter(nn.Module):
    def __init__(self, d_model: int, n_experts: int, group_sizes: list[int] | None = None, k: int = 2,
                 temperature: float = 1.0, jitter_noise: float = 0.0):
        super().__init__()
        self.n_experts, self.k = n_experts, k
        self.temperature, self.jitter_noise = max(1e-6, temperature), jitter_noise
        self.group_sizes = list(group_sizes) if group_sizes else []
        self.gate_group = nn.Linear(d_model, max(1, len(self.group_sizes)), bias=False)
        self.gate_expert = nn.Linear(d_model, n_experts, bias=False)
        self.cond_proj = nn.Linear(2 * d_model, d_model, bias=False)
        self.ranges, s = [], 0
        for g in self.group_sizes:
            self.ranges.append((s, min(n_experts, s + g)))
            s += g

    def forward(self, x: torch.Tensor, cond: dict | None = None):
        h = x
        if cond:
            for key in ("text", "image", "audio", "video"):
                c = cond.get(key)
                if isinstance(c, torch.Tensor) and c.dim() == 2 and c.shape[0] == x.shape[0]:
                    h = self.cond_proj(torch.cat([x, c[:, None].expand(-1, x.shape[1], -1)], -1))
                    break
        logits = self.gate_expert(h)
        if self.training and self.jitter_noise > 0:
            logits = logits + self.jitter_noise * torch.randn_like(logits)
        if self.ranges:
            gsel = torch.softmax(self.gate_group(h), -1).argmax(-1)           # [B, T]
            e = torch.arange(self.n_experts, device=x.device)
            lo = torch.tensor([a for a, _ in self.ranges], device=x.device)[gsel][..., None]
            hi = torch.tensor([b for _, b in self.ranges], device=x.device)[gsel][..., None]
            logits = logits.masked_fill((e < lo) | (e >= hi), -1e9)
        logits = logits / self.temperature
        probs = torch.softmax(logits, -1)
        vals, idx = torch.topk(logits, self.k, -1)
        return idx, torch.softmax(vals, -1), probs, _aux_stats(probs, idx, None, self.n_experts)


class MultiHeadRouter(nn.Module):
    def __init__(self, d_model: int, n_experts: int, k: int = 2, num_gates: int = 4, temperature: float = 1.0,
                 jitter_noise: float = 0.0):
        super().__init__()
        self.n_experts, self.k = n_experts, k
        self.temperature, self.jitter_noise = max(1e-6, temperature), jitter_noise
        self.gates = nn.ModuleList([nn.Linear(d_model, n_experts, bias=False) for _ in range(max(1, num_gates))])

    def forward(self, x: torch.Tensor):
        acc = 0
        for g in self.gates:
            lg = g(x)
            if self.training and self.jitter_noise > 0:
                lg = lg + self.jitter_noise * torch.randn_like(lg)
            acc = acc + torch.softmax(lg / self.temperature, -1)
        probs = acc / len(self.gates)
        vals, idx = torch.topk(probs, self.k, -1)
        scores = vals / vals.sum(-1, keepdim=True).clamp_min(1e-9)
        aux = {"importance": probs.reshape(-1, self.n_experts).mean(0).detach(),
               "load": (probs > 0).to(probs.dtype).reshape(-1, self.n_experts).mean(0).detach()}
        return idx, scores, probs, aux


class GRINGate(nn.Module):
    def __init__(self, d_model: int, n_experts: int, k: int = 2, temperature: float = 1.0, jitter_noise: float = 0.0,
                 mask_drop: float = 0.0):
        super().__init__()
        self.n_experts, self.k = n_experts, k
        self.temperature, self.jitter_noise, self.mask_drop = max(1e-6, temperature), jitter_noise, mask_drop
        self.base_gate = nn.Linear(d_model, n_experts, bias=False)
        self.diff_pred = nn.Sequential(nn.LayerNorm(d_model), nn.Linear(d_model, d_model // 2, bias=False), nn.GELU(),
                                       nn.Linear(d_model // 2, 1, bias=False))

    def forward(self, x: torch.Tensor):
        logits = self.base_gate(x) / (1.0 + torch.sigmoid(self.diff_pred(x)))
        if self.training and self.jitter_noise > 0:
            logits = logits + self.jitter_noise * torch.randn_like(logits)
        logits = logits / self.temperature
        if self.training and self.mask_drop > 0:
            logits = logits.masked_fill(torch.rand_like(logits) < self.mask_drop, -1e9)
        soft = torch.softmax(logits, -1)
        _, idx = torch.topk(logits, self.k, -1)
        hard = F.one_hot(idx, self.n_experts).to(soft.dtype).amax(-2)
        st = hard - soft.detach() + soft                                      # straight-through
        scores = st.gather(-1, idx)
        scores = scores / scores.sum(-1, keepdim=True).clamp_min(1e-9)
        aux = {"importance": soft.reshape(-1, self.n_experts).mean(0).detach(),
               "load": hard.reshape(-1, self.n_experts).mean(0).detach()}
        return idx, scores, soft, aux


class LLMRouter(nn.Module):
    def __init__(self, d_model: int, n_experts: int, k: int = 2, temperature: float = 1.0, jitter_noise: float = 0.0,
                 num_heads: int = 4):
        super().__init__()
        self.n_experts, self.k = n_experts, k
        self.temperature, self.jitter_noise = max(1e-6, temperature), jitter_noise
        self.ln = nn.LayerNorm(d_model)
        self.attn = nn.MultiheadAttention(d_model, num_heads=max(1, num_heads), batch_first=True)
        self.ff = nn.Sequential(nn.Linear(d_model, 2 * d_model, bias=False), nn.GELU(),
                                nn.Linear(2 * d_model, d_model, bias=False))
        self.gate = nn.Linear(d_model, n_experts, bias=False)

    def forward(self, x: torch.Tensor):
        h = self.ln(x)
        t = h.shape[1]
        mask = torch.triu(torch.ones(t, t, dtype=torch.bool, device=x.device), 1)
        h2 = h + self.attn(h, h, h, attn_mask=mask, need_weights=False)[0]
        logits = self.gate(h2 + self.ff(h2))
        if self.training and self.jitter_noise > 0:
            logits = logits + self.jitter_noise * torch.randn_like(logits)
        logits = logits / self.temperature
        probs = torch.softmax(logits, -1)
        vals, idx = torch.topk(logits, self.k, -1)
        return idx, torch.softmax(vals, -1), probs, _aux_stats(probs, idx, logits, self.n_experts)


class InteractionRouter(nn.Module):
    """Gate over cond_proj([x, condition]) when a conditioning embedding (B, C) is
    given (image / text / audio / video, first found), plain top-k gate otherwise
    (reference routing.py:537-600)."""

    def __init__(self, d_model: int, n_experts: int, k: int = 2, temperature: float = 1.0):
        super().__init__()
        self.n_experts, self.k, self.temperature = n_experts, k, max(1e-6, temperature)
        self.gate = nn.Linear(d_model, n_experts, bias=False)
        self.cond_proj = nn.Linear(2 * d_model, d_model, bias=False)

    def forward(self, x: torch.Tensor, cond: dict | None = None):
        h = x
        if cond:
            for key in ("image", "text", "audio", "video"):
                c = cond.get(key)
                if isinstance(c, torch.Tensor) and c.dim() == 2 and c.shape[0] == x.shape[0]:
                    h = self.cond_proj(torch.cat([x, c[:, None].expand(-1, x.shape[1], -1)], -1))
                    break
        logits = self.gate(h) / self.temperature
        probs = torch.softmax(logits, -1)
        vals, idx = torch.topk(logits, self.k, -1)
        return idx, torch.softmax(vals, -1), probs, _aux_stats(probs, idx, logits, self.n_experts)


def load_balance_loss(aux: dict, n_experts: int) -> torch.Tensor:
    """Switch-style balance term E * sum_e importance_e * load_e."""
    return n_experts * (aux["importance"] * aux["load"]).sum()


# ----------------------------------------------------------------------------
# HRM: planner / worker GRUs (reference src/omnicoder/modeling/hrm.py)
# ----------------------------------------------------------------------------
class Planner(nn.Module):
    def __init__(self, d_model: int):
        super().__init__()
        self.rnn = nn.GRU(d_model, d_model, batch_first=True)
        self.policy = nn.Linear(d_model, d_model)

    def forward(self, state, h=None):
        out, h = self.rnn(state, h)
        return self.policy(out[:, -1:]), h


class Worker(nn.Module):
    def __init__(self, d_model: int):
        super().__init__()
        self.rnn = nn.GRU(d_model, d_model, batch_first=True)
        self.act = nn.Linear(d_model, d_model)

    def forward(self, state, intent, h=None):
        out, h = self.rnn(state + intent.expand(-1, state.shape[1], -1), h)
        return self.act(out), h


class HRM(nn.Module):
    """`steps` rounds of: planner GRU over the sequence -> intent (last step) ->
    worker GRU over (state + intent).  With adaptive halting, a halting head
    accumulates per-token continuation probability and tokens stop updating once
    the sum crosses the threshold (ACT-style)."""

    def __init__(self, d_model: int, steps: int = 3, adaptive_halting: bool = False, halting_threshold: float = 0.99,
                 max_steps_budget: int | None = None):
        super().__init__()
        self.planner, self.worker = Planner(d_model), Worker(d_model)
        self.steps = max(1, steps)
        self.adaptive_halting, self.halting_threshold = adaptive_halting, halting_threshold
        self.max_steps_budget = max_steps_budget
        self.halt_head = nn.Sequential(nn.LayerNorm(d_model), nn.Linear(d_model, d_model // 2), nn.GELU(),
                                       nn.Linear(d_model // 2, 1)) if adaptive_halting else None

    def forward(self, state: torch.Tensor) -> torch.Tensor:
        n = self.steps if not self.max_steps_budget else min(self.steps, self.max_steps_budget)
        hp = hw = None
        if not self.adaptive_halting:
            for _ in range(n):
                intent, hp = self.planner(state, hp)
                state, hw = self.worker(state, intent, hw)
            return state
        acc = state.new_zeros(*state.shape[:-1], 1)
        for _ in range(n):
            intent, hp = self.planner(state, hp)
            new, hw = self.worker(state, intent, hw)
            p = torch.sigmoid(self.halt_head(new))
            running = (acc < self.halting_threshold).to(state.dtype)
            state = running * new + (1 - running) * state
            acc = acc + p * running
        return state


# ----------------------------------------------------------------------------
# Memory (reference src/omnicoder/modeling/memory.py)
# ----------------------------------------------------------------------------
class RecurrentMemory(nn.Module):
    """M learned slot queries attend over the hidden states; the result is
    blended 50/50 with the mean state and passed through a small MLP."""

    def __init__(self, d_model: int, num_slots: int = 8, reduce: str = "mean"):
        super().__init__()
        self.num_slots, self.reduce = max(1, num_slots), reduce
        self.slot_query = nn.Parameter(torch.randn(self.num_slots, d_model) * 0.02)
        self.post = nn.Sequential(nn.LayerNorm(d_model), nn.Linear(d_model, d_model), nn.GELU(),
                                  nn.Linear(d_model, d_model))

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        att = torch.softmax(torch.einsum("mc,btc->bmt", self.slot_query, hidden) / math.sqrt(hidden.shape[-1]), -1)
        mem = torch.einsum("bmt,btc->bmc", att, hidden)
        if self.reduce == "mean":
            mem = 0.5 * mem + 0.5 * hidden.mean(1, keepdim=True)
        return self.post(mem)


class CompressiveKV(nn.Module):
    """Compress a latent K/V prefix [B, H, T, DL] into `slots` segment summaries:
    segment mean x sigmoid(write gate) x retention scale (keep + 0.5 compress of
    a 3-way softmax), then LayerNorm + Linear per stream."""

    def __init__(self, latent_dim: int, slots: int = 8):
        super().__init__()
        self.slots = max(1, slots)
        self.post_k = nn.Sequential(nn.LayerNorm(latent_dim), nn.Linear(latent_dim, latent_dim, bias=False))
        self.post_v = nn.Sequential(nn.LayerNorm(latent_dim), nn.Linear(latent_dim, latent_dim, bias=False))
        self.write_gate = nn.Sequential(nn.LayerNorm(latent_dim), nn.Linear(latent_dim, 1))
        self.retention_head = nn.Sequential(nn.LayerNorm(latent_dim), nn.Linear(latent_dim, 3))

    def segments(self, T: int) -> list[tuple[int, int]]:
        base, rem = divmod(max(T, 0), self.slots)
        out, s = [], 0
        for i in range(self.slots):
            e = s + base + (1 if i < rem else 0)
            out.append((s, e))
            s = e
        return out

    def forward(self, k_lat: torch.Tensor, v_lat: torch.Tensor):
        ks, vs = [], []
        for a, b in self.segments(k_lat.shape[2]):
            if b <= a:
                ks.append(k_lat.new_zeros(*k_lat.shape[:2], 1, k_lat.shape[-1]))
                vs.append(v_lat.new_zeros(*v_lat.shape[:2], 1, v_lat.shape[-1]))
                continue
            k = k_lat[:, :, a:b].mean(2, keepdim=True)
            v = v_lat[:, :, a:b].mean(2, keepdim=True)
            g = torch.sigmoid(self.write_gate(k))
            p = torch.softmax(self.retention_head(k * g), -1)
            scale = g * (p[..., 0:1] + 0.5 * p[..., 1:2])
            ks.append(k * scale)
            vs.append(v * scale)
        return self.post_k(torch.cat(ks, 2)), self.post_v(torch.cat(vs, 2))


def compressive_aux_loss(mem: torch.Tensor, hidden: torch.Tensor, reduce: bool = True) -> torch.Tensor:
    """1 - cosine(slot, mean hidden state), averaged (reference memory.py:181-193)."""
    cos = (F.normalize(mem, dim=-1) * F.normalize(hidden.mean(1, keepdim=True), dim=-1)).sum(-1)
    loss = (1 - cos).mean(-1)
    return loss.mean() if reduce else loss


class LandmarkIndexer(nn.Module):
    """`num_landmarks` learned queries attend over the sequence; post MLP."""

    def __init__(self, d_model: int, num_landmarks: int = 8):
        super().__init__()
        self.num_landmarks = max(1, num_landmarks)
        self.query = nn.Parameter(torch.randn(self.num_landmarks, d_model) * 0.02)
        self.post = nn.Sequential(nn.LayerNorm(d_model), nn.Linear(d_model, d_model), nn.GELU(),
                                  nn.Linear(d_model, d_model))

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        att = torch.softmax(torch.einsum("mc,btc->bmt", self.query, hidden) / math.sqrt(hidden.shape[-1]), -1)
        return self.post(torch.einsum("bmt,btc->bmc", att, hidden))


# ----------------------------------------------------------------------------
# Sequence mixers (reference ssm.py, hyena.py)
# ----------------------------------------------------------------------------
class GatedMambaSSM(nn.Module):
    """in_proj -> depthwise conv (k=7, same padding) -> x sigmoid(gate(x)) -> out."""

    def __init__(self, d_model: int, expansion: int = 2, kernel_size: int = 7):
        super().__init__()
        h = d_model * expansion
        self.in_proj = nn.Linear(d_model, h, bias=False)
        self.conv = nn.Conv1d(h, h, kernel_size, padding=kernel_size // 2, groups=h)
        self.gate = nn.Linear(d_model, h, bias=False)
        self.out = nn.Linear(h, d_model, bias=False)

    def forward(self, x):
        h = self.conv(self.in_proj(x).transpose(1, 2)).transpose(1, 2)
        return self.out(h * torch.sigmoid(self.gate(x)))


class GatedConvSSM(nn.Module):
    """LayerNorm -> GLU(u * gelu(v)) -> depthwise conv -> projection."""

    def __init__(self, d_model: int, kernel_size: int = 7, expansion: int = 2, dropout_p: float = 0.0):
        super().__init__()
        h = d_model * expansion
        self.norm = nn.LayerNorm(d_model)
        self.proj_in = nn.Linear(d_model, 2 * h, bias=False)
        self.dw_conv = nn.Conv1d(h, h, kernel_size, groups=h, padding=kernel_size // 2)
        self.proj_out = nn.Linear(h, d_model, bias=False)
        self.dropout = nn.Dropout(dropout_p) if dropout_p > 0 else nn.Identity()

    def forward(self, x):
        u, v = self.proj_in(self.norm(x)).chunk(2, -1)
        y = self.dw_conv((u * F.gelu(v)).transpose(1, 2)).transpose(1, 2)
        return self.dropout(self.proj_out(y))


class HyenaMixer1D(nn.Module):
    """Causal long depthwise convolution with symmetric cross gating:
    u = in(x) split in halves a, b; A = conv_a(a), B = conv_b(b) (left padding of
    kernel_size - 1 keeps them causal); y = out([A * sigmoid(B), B * sigmoid(A)])."""

    def __init__(self, hidden_dim: int, expansion: int = 2, kernel_size: int = 256, depthwise: bool = True):
        super().__init__()
        c = hidden_dim * expansion
        half = c // 2
        self.kernel_size = kernel_size
        self.in_proj = nn.Conv1d(hidden_dim, c, 1)
        self.long_conv_a = nn.Conv1d(half, half, kernel_size, groups=half if depthwise else 1)
        self.long_conv_b = nn.Conv1d(half, half, kernel_size, groups=half if depthwise else 1)
        self.out_proj = nn.Conv1d(c, hidden_dim, 1)

    def forward(self, x):
        u = self.in_proj(x.transpose(1, 2))
        a, b = u.chunk(2, 1)
        pad = (self.kernel_size - 1, 0)
        A = self.long_conv_a(F.pad(a, pad))
        B = self.long_conv_b(F.pad(b, pad))
        return self.out_proj(torch.cat([A * torch.sigmoid(B), B * torch.sigmoid(A)], 1)).transpose(1, 2)


# ----------------------------------------------------------------------------
# Expert FFN of the reference (experts.py): fc1 -> GELU(tanh) (or SiLU) -> fc2, with biases
# ----------------------------------------------------------------------------
class ExpertFFN(nn.Module):
    def __init__(self, d_model: int, mlp_dim: int, act: str = "gelu"):
        super().__init__()
        self.fc1 = nn.Linear(d_model, mlp_dim)
        self.fc2 = nn.Linear(mlp_dim, d_model)
        self.act = act

    def forward(self, x):
        h = self.fc1(x)
        h = F.silu(h) if self.act == "silu" else F.gelu(h, approximate="tanh")
        return self.fc2(h)
