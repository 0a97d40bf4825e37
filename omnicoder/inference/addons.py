"""Decode-time add-ons of :func:`omnicoder.inference.generate.generate`.

Each add-on changes the next-token logits of a decode step (or a decision of
the speculative loop) from quantities the step already has on the device: the
last position's logits [B, V] and final hidden state [B, D].  None of them
reads the host inside a step unless its decision is a host decision by nature
(adaptive expert count, early exit).

  * kNN-LM blend (reference src/omnicoder/inference/generate.py:2085-2136):
    p = (1 - lambda) softmax(logits) + lambda p_knn(hidden); the step's
    (hidden, argmax token) pair is written to the cache every `write_every` steps.
  * retrieval bias (:2784-2821): retrieved texts are embedded as the mean of
    their token embeddings, attended by the last hidden state
    (softmax(h . r / sqrt(D))), and the attended vector's head logits are added
    with weight alpha.
  * structured factor bias (SFB, :835-976): the prompt is factorised into
    sub-goals; the tokens of each goal vote with the goal's weight and the
    mixture becomes an additive log-bias (omnicoder.reasoning.sfb.cross_bias).
  * dual substrate (:2053-2083): when the model carries a byte head, its logits
    are blended in with gate sigmoid(alpha * entropy + beta * KL(p_model || p_byte)).
  * adaptive expert count (:2405-2432): the routed experts per token of every MoE
    layer follow the step's confidence (max probability): `k_max` below
    `conf_floor`, `k_min` above it.
  * early exit (:2433-2467): a confident step (entropy <= threshold, or top-1
    minus top-2 logit >= threshold) skips the speculative draft.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


def _entropy(logits: torch.Tensor) -> torch.Tensor:
    p = torch.softmax(logits.float(), -1)
    return -(p * torch.log(p.clamp_min(1e-9))).sum(-1)


@dataclass
class DecodeAddons:
    knn_cache: object | None = None
    knn_k: int = 16
    knn_lambda: float = 0.2
    knn_write_every: int = 8
    retrieval_vecs: torch.Tensor | None = None      # [N, D] mean token embeddings of retrieved texts
    retrieval_alpha: float = 0.0
    sfb_bias: torch.Tensor | None = None            # [V] additive log-bias
    sfb_alpha: float = 1.0
    dual_alpha: float = 1.0
    dual_beta: float = 1.0
    dual: bool = False
    steps: int = field(default=0)

    @property
    def needs_hidden(self) -> bool:
        return (self.knn_cache is not None and self.knn_lambda > 0) or self.retrieval_vecs is not None or self.dual

    @property
    def active(self) -> bool:
        return self.needs_hidden or self.sfb_bias is not None

    @torch.no_grad()
    def apply(self, model, logits: torch.Tensor, hidden: torch.Tensor | None) -> torch.Tensor:
        """logits [B, V], hidden [B, D] of the same position -> adjusted logits [B, V] (fp32)."""
        x = logits.float()
        h = hidden.reshape(x.shape[0], -1).float() if hidden is not None else None
        if self.retrieval_vecs is not None and h is not None and self.retrieval_alpha > 0:
            r = self.retrieval_vecs.float()
            w = torch.softmax(h @ r.t() / max(1.0, math.sqrt(h.shape[-1])), dim=-1)
            ctx = (w @ r).to(model.head_weight.dtype)
            x = x + self.retrieval_alpha * (ctx @ model.head_weight.t()).float()
        if self.dual and h is not None and getattr(model, "byte_head", None) is not None:
            bl = (h.to(model.byte_head.dtype) @ model.byte_head.t()).float()
            lp, lb = torch.log_softmax(x, -1), torch.log_softmax(bl, -1)
            ent = -(lp.exp() * lp).sum(-1, keepdim=True)
            kl = (lp.exp() * (lp - lb)).sum(-1, keepdim=True)
            g = torch.sigmoid(self.dual_alpha * ent + self.dual_beta * kl)
            x = (1.0 - g) * x + g * bl
        if self.sfb_bias is not None:
            x = x + self.sfb_alpha * self.sfb_bias
        if self.knn_cache is not None and self.knn_lambda > 0 and h is not None:
            cache = self.knn_cache
            if self.knn_write_every > 0 and self.steps % self.knn_write_every == 0:
                cache.add(h, x.argmax(-1))
            if len(cache):
                k_old = cache.k
                cache.k = max(1, int(self.knn_k))
                p_knn = cache.query(h, x.shape[-1])
                cache.k = k_old
                p = (1.0 - self.knn_lambda) * torch.softmax(x, -1) + self.knn_lambda * p_knn
                x = torch.log(p.clamp_min(1e-8))
        self.steps += 1
        return x


def retrieval_vectors(model, texts: list[str], encode_fn, max_texts: int = 8) -> torch.Tensor | None:
    """Mean token embedding of each retrieved text ([N, D] on the model's device)."""
    vecs = []
    emb = model.embed
    for t in texts[:max_texts]:
        ids = [int(i) for i in encode_fn(t) if 0 <= int(i) < emb.shape[0]]
        if ids:
            vecs.append(emb[torch.tensor(ids, device=emb.device)].float().mean(0))
    return torch.stack(vecs) if vecs else None


def sfb_token_bias(prompt_text: str, encode_fn, vocab: int, device, strength: float = 1.0) -> torch.Tensor | None:
    """Structured factor bias (omnicoder.sfb.sfb_bias): the prompt is factorised, belief
    propagation over its goal families weights each sub-goal, and the weighted token
    distributions of the goals' strings become an additive log-bias relative to uniform."""
    from ..sfb import sfb_bias
    return sfb_bias(prompt_text, encode_fn, vocab, device, strength=strength)


def adapt_moe_top_k(model, logits: torch.Tensor, k_min: int, k_max: int, conf_floor: float,
                    layer_ramp: bool = False, layer_power: float = 1.0) -> int:
    """Set the routed experts per token of every MoE layer from the step's confidence (mean over
    the batch of the max next-token probability; one host read).  With `layer_ramp` early
    layers keep more experts than late ones.  Returns the chosen k."""
    from ..models.lm import MoEFFN
    conf = float(torch.softmax(logits.float(), -1).max(-1).values.mean())
    k = int(k_max if conf < conf_floor else k_min)
    moes = [b.ffn for b in model.blocks if isinstance(b.ffn, MoEFFN)]
    L = len(moes)
    for li, m in enumerate(moes):
        kl = k
        if layer_ramp and L > 1:
            frac = 1.0 - li / (L - 1)
            kl = max(1, int(round(1 + (k - 1) * max(0.0, min(1.0, frac)) ** max(0.0, layer_power))))
        m.top_k_override = max(1, min(kl, model.cfg.moe.n_experts))
    return k


def clear_moe_top_k(model):
    from ..models.lm import MoEFFN
    for b in model.blocks:
        if isinstance(b.ffn, MoEFFN):
            b.ffn.top_k_override = None


def confident(logits: torch.Tensor, mode: str, threshold: float) -> bool:
    """Early-exit test of a decode step (all sequences of the batch): entropy <= threshold, or
    top-1 minus top-2 logit >= max(threshold, 1)."""
    x = logits.float()
    if mode == "entropy":
        return bool((_entropy(x) <= threshold).all())
    if mode == "delta":
        t2 = torch.topk(x, 2, dim=-1).values
        return bool(((t2[..., 0] - t2[..., 1]) >= max(threshold, 1.0)).all())
    raise ValueError(f"unknown early-exit mode {mode!r}")
