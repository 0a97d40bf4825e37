"""Expert-level utilities of the reference, restated.

* ExpertPager (reference modeling/utils/expert_paging.py:13-191): an LRU of
  expert modules materialised on demand from factories, optionally persisted to
  disk, with explicit and background prefetch and a routing-probability hint.
* upcycle_ffn_to_experts (utils/cumo.py:7-66): grow every MoE expert list to
  `target_experts` by cloning expert 0 with small Gaussian perturbations
  (co-upcycling a dense FFN into experts).
* HyperExpertSynthesizer (hyper_expert.py:21-84): an MLP that maps a
  conditioning vector to the full weights of one FFN expert.
* PerceiverIOTower (perceiver_io.py:8-66): latent array cross-attends to the
  inputs, self-attention blocks over the latents, pooled back to the input
  length.
* DiffusionTextGenerator (diffusion_text.py:20-211): embedding-space diffusion
  decoding over a cosine schedule with the LM as denoiser; tokens are the
  nearest embeddings of the final estimate.
"""
from __future__ import annotations

import collections
import copy
import math
import os
import threading
from dataclasses import dataclass
from typing import Callable

import torch
import torch.nn as nn
import torch.nn.functional as F


class ExpertPager:
    def __init__(self, capacity: int = 8, device=None, persist_dir: str | None = None):
        self.capacity = max(1, capacity)
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.persist_dir = persist_dir
        self.factories: dict[int, Callable[[], nn.Module]] = {}
        self.resident: "collections.OrderedDict[int, nn.Module]" = collections.OrderedDict()
        self.hits = self.misses = self.evictions = 0
        self._lock = threading.Lock()
        self._queue: list[int] = []
        self._worker: threading.Thread | None = None

    def register(self, idx: int, factory: Callable[[], nn.Module]) -> None:
        self.factories[idx] = factory

    def _path(self, idx: int) -> str | None:
        return None if self.persist_dir is None else os.path.join(self.persist_dir, f"expert_{idx}.pt")

    def _materialise(self, idx: int) -> nn.Module:
        m = self.factories[idx]()
        p = self._path(idx)
        if p is not None and os.path.exists(p):
            m.load_state_dict(torch.load(p, map_location="cpu"))
        return m.to(self.device)

    def get(self, idx: int) -> nn.Module:
        with self._lock:
            if idx in self.resident:
                self.hits += 1
                self.resident.move_to_end(idx)
                return self.resident[idx]
            self.misses += 1
        m = self._materialise(idx)
        with self._lock:
            self.resident[idx] = m
            self.resident.move_to_end(idx)
            while len(self.resident) > self.capacity:
                old, mod = self.resident.popitem(last=False)
                p = self._path(old)
                if p is not None:
                    os.makedirs(self.persist_dir, exist_ok=True)
                    torch.save(mod.state_dict(), p)
                self.evictions += 1
        return m

    def prefetch(self, indices: list[int]) -> None:
        for i in indices:
            if i in self.factories:
                self.get(i)

    def request_prefetch(self, indices: list[int]) -> None:
        """Prefetch on a background thread."""
        with self._lock:
            self._queue.extend(i for i in indices if i not in self.resident)
        if self._worker is None or not self._worker.is_alive():
            def run():
                while True:
                    with self._lock:
                        if not self._queue:
                            return
                        i = self._queue.pop(0)
                    self.get(i)
            self._worker = threading.Thread(target=run, daemon=True)
            self._worker.start()

    def warm_hint(self, probs: torch.Tensor, topk: int = 2) -> None:
        """Prefetch the experts with the highest mean routing probability."""
        mean = probs.reshape(-1, probs.shape[-1]).float().mean(0)
        self.request_prefetch(torch.topk(mean, min(topk, mean.numel())).indices.tolist())

    def stats(self) -> dict:
        return {"resident": list(self.resident), "hits": self.hits, "misses": self.misses,
                "evictions": self.evictions, "capacity": self.capacity}


@torch.no_grad()
def upcycle_ffn_to_experts(module: nn.Module, target_experts: int, noise_std: float = 1e-3) -> int:
    """Returns the number of MoE layers that were grown."""
    grown = 0
    for child in module.modules():
        experts = getattr(child, "experts", None)
        if not isinstance(experts, nn.ModuleList) or len(experts) == 0 or len(experts) >= target_experts:
            continue
        base = experts[0]
        new = nn.ModuleList()
        for i in range(target_experts):
            e = copy.deepcopy(base)
            if i > 0:
                for p in e.parameters():
                    p.add_(torch.randn_like(p) * noise_std)
            new.append(e)
        child.experts = new
        if hasattr(child, "n_experts"):
            child.n_experts = target_experts
        grown += 1
    return grown


@dataclass
class HyperExpertSpec:
    d_model: int
    mlp_dim: int


class HyperExpertSynthesizer(nn.Module):
    def __init__(self, spec: HyperExpertSpec, cond_dim: int = 512, hidden: int = 1024):
        super().__init__()
        self.spec = spec
        d, m = spec.d_model, spec.mlp_dim
        self.net = nn.Sequential(nn.LayerNorm(cond_dim), nn.Linear(cond_dim, hidden), nn.GELU(),
                                 nn.Linear(hidden, hidden), nn.GELU(), nn.Linear(hidden, 2 * d * m + m + d))

    def forward(self, cond: torch.Tensor) -> dict:
        """cond [B, cond_dim] -> {'w1': [B, m, d], 'b1': [B, m], 'w2': [B, d, m], 'b2': [B, d]}."""
        d, m = self.spec.d_model, self.spec.mlp_dim
        v = self.net(cond)
        w1, b1, w2, b2 = torch.split(v, [d * m, m, m * d, d], dim=-1)
        B = cond.shape[0]
        return {"w1": w1.reshape(B, m, d), "b1": b1, "w2": w2.reshape(B, d, m), "b2": b2}

    @staticmethod
    def apply(weights: dict, x: torch.Tensor, i: int = 0) -> torch.Tensor:
        """Run synthesised expert i on x [T, d] (GELU-tanh FFN)."""
        h = F.gelu(x @ weights["w1"][i].t() + weights["b1"][i], approximate="tanh")
        return h @ weights["w2"][i].t() + weights["b2"][i]


def serialize_synthesized(weights: dict, path: str) -> None:
    torch.save({k: v.detach().cpu() for k, v in weights.items()}, path)


class PerceiverIOTower(nn.Module):
    def __init__(self, d_io: int = 128, d_latent: int = 256, n_latents: int = 64, n_layers: int = 4, n_heads: int = 8):
        super().__init__()
        self.d_latent = d_latent
        self.latents = nn.Parameter(torch.randn(n_latents, d_latent) * 0.02)
        self.q_proj = nn.Linear(d_latent, d_latent, bias=False)
        self.k_proj = nn.Linear(d_io, d_latent, bias=False)
        self.v_proj = nn.Linear(d_io, d_latent, bias=False)
        self.sa_layers = nn.ModuleList([nn.ModuleDict({
            "ln1": nn.LayerNorm(d_latent), "qkv": nn.Linear(d_latent, 3 * d_latent, bias=False),
            "proj": nn.Linear(d_latent, d_latent, bias=False), "ln2": nn.LayerNorm(d_latent),
            "mlp": nn.Sequential(nn.Linear(d_latent, 4 * d_latent), nn.GELU(), nn.Linear(4 * d_latent, d_latent)),
        }) for _ in range(n_layers)])
        self.to_io = nn.Linear(d_latent, d_io, bias=False)

    def forward(self, io: torch.Tensor) -> torch.Tensor:
        B, T, _ = io.shape
        sc = 1.0 / math.sqrt(self.d_latent)
        lat = self.latents[None].expand(B, -1, -1)
        a = torch.softmax(self.q_proj(lat) @ self.k_proj(io).transpose(1, 2) * sc, -1)
        lat = lat + a @ self.v_proj(io)
        for blk in self.sa_layers:
            q, k, v = blk["qkv"](blk["ln1"](lat)).chunk(3, -1)
            lat = lat + blk["proj"](torch.softmax(q @ k.transpose(1, 2) * sc, -1) @ v)
            lat = lat + blk["mlp"](blk["ln2"](lat))
        return self.to_io(lat.mean(1, keepdim=True).expand(B, T, -1))


def cosine_schedule(steps: int, device=None):
    """(betas, sqrt(abar), sqrt(1 - abar)) of the cosine schedule abar_t = cos^2(pi/2 (t + 0.008)/(T + 0.008))."""
    t = torch.arange(steps, dtype=torch.float32, device=device)
    abar = torch.cos((t + 0.008) / (steps + 0.008) * math.pi / 2) ** 2
    prev = torch.cat([abar[:1], abar[:-1]]).clamp_min(1e-5)
    return 1 - abar / prev, abar.sqrt(), (1 - abar).sqrt()


class DiffusionTextGenerator(nn.Module):
    """`denoise(emb [B, T, D]) -> emb` is the model run on embeddings (for the spec
    family: the blocks without the embedding lookup); tokens are read out by
    nearest neighbour against the embedding matrix."""

    def __init__(self, denoise: Callable[[torch.Tensor], torch.Tensor], embed: torch.Tensor, num_steps: int = 8):
        super().__init__()
        D = embed.shape[1]
        self.denoise, self.embed, self.num_steps = denoise, embed, max(1, num_steps)
        self.t_embed = nn.Sequential(nn.Linear(D, D), nn.SiLU(), nn.Linear(D, D))
        self.register_buffer("time_w", torch.linspace(1.0, 1000.0, D), persistent=False)

    @torch.no_grad()
    def generate(self, prompt_ids: torch.Tensor | None, gen_tokens: int, steps: int | None = None,
                 generator: torch.Generator | None = None) -> torch.Tensor:
        n = steps or self.num_steps
        E = self.embed.float()
        B = 1 if prompt_ids is None else prompt_ids.shape[0]
        prompt = E[prompt_ids] if prompt_ids is not None else E.new_zeros(B, 0, E.shape[1])
        x = torch.randn(B, gen_tokens, E.shape[1], generator=generator, device=E.device)
        _, sa, s1a = cosine_schedule(n, E.device)
        for i in range(n - 1, -1, -1):
            r = i / max(1, n - 1)
            te = self.t_embed(torch.sin(r * self.time_w)).to(x.dtype)
            h = self.denoise(torch.cat([prompt, x + te], 1))[:, prompt.shape[1]:].float()
            x0 = h
            if i > 0:
                noise = torch.randn(x.shape, generator=generator, device=x.device)
                x = sa[i - 1] * x0 + s1a[i - 1] * noise
            else:
                x = x0
        dist = (x[..., None, :] - E[None, None]).pow(2).sum(-1) if E.shape[0] * gen_tokens < 4_000_000 else None
        return dist.argmin(-1) if dist is not None else (x @ E.t()).argmax(-1)
