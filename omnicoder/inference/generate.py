"""Batched text generation: prefill + KV-cache decode, sampling, speculative decoding.

Public API (same entry point as the reference, src/omnicoder/inference/generate.py:692):

    generate(model, input_ids, max_new_tokens, temperature=0.8, top_k=40, top_p=0.9,
             draft_model=None, speculative_draft_len=0, kvq="none", window_size=0,
             return_stats=False, eos_id=None, seed=None)

Differences from the reference, by design:
  * batched (B >= 1) prefill of the whole prompt (the reference feeds only the last
    prompt token, with B == 1);
  * temperature <= 0 means greedy decoding (the reference clamps temperature to >= 0.2);
  * speculative decoding verifies all draft tokens in one target forward and accepts
    them by rejection sampling (exact-match when greedy), so the output distribution
    is the target's; the reference accepts by a verifier-probability threshold and
    re-feeds accepted tokens one at a time (generate.py:2925-3048);
  * `kvq="int8"` stores the cache as int8 with per-token (MLA) / per-head-per-token
    (MHA/GQA) scales.
"""
from __future__ import annotations

import argparse
import json
import sys
import time
from dataclasses import dataclass, field

import torch

from .kv_cache import KVCache


# ----------------------------------------------------------------------------
# Sampling
# ----------------------------------------------------------------------------
def _filter_logits(logits: torch.Tensor, top_k: int, top_p: float) -> torch.Tensor:
    logits = torch.where(torch.isfinite(logits), logits, torch.full_like(logits, float("-inf")))
    if top_k and top_k > 0 and top_k < logits.shape[-1]:
        kth = torch.topk(logits, top_k, dim=-1).values[..., -1:]
        logits = logits.masked_fill(logits < kth, float("-inf"))
    if top_p is not None and 0.0 < top_p < 1.0:
        sorted_logits, idx = torch.sort(logits, dim=-1, descending=True)
        probs = torch.softmax(sorted_logits, dim=-1)
        cum = probs.cumsum(-1)
        remove = cum - probs > top_p
        sorted_logits = sorted_logits.masked_fill(remove, float("-inf"))
        logits = torch.full_like(logits, float("-inf")).scatter(-1, idx, sorted_logits)
    return logits


def sampling_probs(logits: torch.Tensor, temperature: float, top_k: int = 0, top_p: float = 1.0) -> torch.Tensor:
    """The distribution that sample_next_token draws from (fp32 [..., V])."""
    logits = logits.float()
    if temperature <= 0:
        return torch.nn.functional.one_hot(logits.argmax(-1), logits.shape[-1]).float()
    return torch.softmax(_filter_logits(logits / temperature, top_k, top_p), dim=-1)


def sample_next_token(logits: torch.Tensor, temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0,
                      generator: torch.Generator | None = None) -> torch.Tensor:
    """logits [..., V] -> token ids [...]; greedy when temperature <= 0."""
    if temperature <= 0:
        return logits.argmax(-1)
    p = sampling_probs(logits, temperature, top_k, top_p)
    flat = p.reshape(-1, p.shape[-1])
    return torch.multinomial(flat, 1, generator=generator).view(p.shape[:-1])


class LogitProcessor:
    """Penalties and biases applied to the logits before sampling (reference
    src/omnicoder/inference/generate.py:500-690 and :2148-2169): CTRL-style repetition penalty
    (the logit of a token seen in the window is divided by `repetition_penalty` when positive
    and multiplied by it when negative), presence / frequency penalties (minus `presence` once
    a token occurred, minus `frequency` x its count) and an additive per-token bias.

    Only the last `window` tokens of each sequence count (default 128, the reference's
    rep_window); `window=0` counts the whole sequence.  Token counts ([B, V]) and the ring of
    the window's token ids ([B, window]) live on the device, so no step reads the host."""

    def __init__(self, batch: int, vocab: int, device, repetition_penalty: float = 1.0, presence_penalty: float = 0.0,
                 frequency_penalty: float = 0.0, logit_bias: dict | None = None, window: int = 128):
        if repetition_penalty <= 0:
            raise ValueError(f"repetition_penalty must be > 0 (got {repetition_penalty})")
        if window < 0:
            raise ValueError(f"penalty window must be >= 0 (got {window})")
        self.rep, self.pres, self.freq = repetition_penalty, presence_penalty, frequency_penalty
        self.vocab = vocab
        self.window = int(window)
        self.counts = torch.zeros(batch, vocab, device=device)
        self.ring = torch.full((batch, self.window), -1, dtype=torch.long, device=device) if self.window else None
        self.head = 0                      # next ring column to overwrite
        self.bias = None
        if logit_bias:
            bad = [t for t in logit_bias if not 0 <= int(t) < vocab]
            if bad:
                raise ValueError(f"logit_bias token ids outside [0, {vocab}): {sorted(bad)[:8]}")
            self.bias = torch.zeros(vocab, device=device)
            for t, b in logit_bias.items():
                self.bias[int(t)] = float(b)

    @property
    def active(self) -> bool:
        return self.rep != 1.0 or self.pres != 0.0 or self.freq != 0.0 or self.bias is not None

    def observe(self, ids: torch.Tensor) -> None:
        """Append the token ids [B, n] (or [B]) of every sequence to the window."""
        ids = ids.reshape(self.counts.shape[0], -1).long()
        one = torch.ones_like(ids[:, :1], dtype=self.counts.dtype)
        if not self.window:
            self.counts.scatter_add_(1, ids, one.expand_as(ids))
            return
        if ids.shape[1] >= self.window:    # the window holds only the newest tokens: rebuild it
            tail = ids[:, -self.window:]
            self.counts.zero_()
            self.counts.scatter_add_(1, tail, one.expand_as(tail))
            self.ring.copy_(tail)
            self.head = 0
            return
        for j in range(ids.shape[1]):
            old = self.ring[:, self.head:self.head + 1]
            # tokens leaving the window (ring slots still -1 subtract nothing)
            self.counts.scatter_add_(1, old.clamp_min(0), -(old >= 0).to(self.counts.dtype))
            new = ids[:, j:j + 1]
            self.counts.scatter_add_(1, new, one)
            self.ring[:, self.head:self.head + 1] = new
            self.head = (self.head + 1) % self.window

    def __call__(self, logits: torch.Tensor) -> torch.Tensor:
        if not self.active:
            return logits
        x = logits.float()
        seen = self.counts > 0
        if self.rep != 1.0:
            x = torch.where(seen, torch.where(x > 0, x / self.rep, x * self.rep), x)
        if self.pres or self.freq:
            x = x - self.pres * seen.float() - self.freq * self.counts
        if self.bias is not None:
            x = x + self.bias
        return x


def load_logit_bias(path: str) -> dict:
    """JSON object {token id: additive bias}."""
    import json
    with open(path) as f:
        return {int(k): float(v) for k, v in json.load(f).items()}


@dataclass
class GenStats:
    prompt_tokens: int = 0
    new_tokens: int = 0
    prefill_s: float = 0.0
    decode_s: float = 0.0
    steps: int = 0
    accepted_draft_tokens: int = 0
    proposed_draft_tokens: int = 0
    early_exits: int = 0
    step_times_s: list = field(default_factory=list)

    @property
    def decode_tokens_per_s(self) -> float:
        return self.new_tokens / self.decode_s if self.decode_s > 0 else 0.0

    def as_dict(self):
        d = {k: v for k, v in self.__dict__.items() if k != "step_times_s"}
        d["decode_tokens_per_s"] = self.decode_tokens_per_s
        if self.step_times_s:
            st = sorted(self.step_times_s)
            d["p50_step_s"] = st[len(st) // 2]
        if self.proposed_draft_tokens:
            d["acceptance_rate"] = self.accepted_draft_tokens / self.proposed_draft_tokens
        return d


PREFILL_TOKENS = 32768   # tokens per prefill call (whole sequences; bounds the activation memory)


def _prefill(model, ids: torch.Tensor, cache, return_hidden: bool = False):
    """Run the prompt through the model in chunks of whole sequences and return the
    last-position logits [B, V] (and final hidden states [B, D] with return_hidden).
    With memory rows and a window, the tokens that left the window are then summarised
    into the memory rows."""
    B, S = ids.shape
    step = max(1, PREFILL_TOKENS // max(1, S))
    out, hid = [], []
    for b0 in range(0, B, step):
        b1 = min(B, b0 + step)
        view = cache.view(b0, b1) if (b0, b1) != (0, B) else cache
        r = model.forward_cached(ids[b0:b1], view, prefill=True, last_only=True, return_hidden=return_hidden)
        if return_hidden:
            out.append(r[0][:, -1])
            hid.append(r[1][:, -1])
        else:
            out.append(r[:, -1])
    cfg = model.cfg
    if getattr(cfg.attn, "mem_slots", 0) and cfg.attn.window:
        cache.compress_memory(cfg.attn.window)
    logits = torch.cat(out) if len(out) > 1 else out[0]
    if return_hidden:
        return logits, (torch.cat(hid) if len(hid) > 1 else hid[0])
    return logits


@torch.no_grad()
def prime_kv_with_features(model, feats: torch.Tensor, cache) -> torch.Tensor:
    """Append feature vectors feats [B, P, D] (e.g. another modality's encoder output, or a
    summary of text beyond the window) to the cache as if they were token embeddings, so the
    following tokens attend to them (reference src/omnicoder/inference/generate.py:1381-1403,
    :3193).  Returns the logits of the last primed position [B, V]."""
    B, P, _ = feats.shape
    ids = torch.zeros(B, P, dtype=torch.long, device=feats.device)
    return model.forward_cached(ids, cache, embeds=feats)[:, -1]


def _sync(t: torch.Tensor):
    if t.is_cuda:
        torch.cuda.synchronize(t.device)


# ----------------------------------------------------------------------------
@torch.no_grad()
def generate(model, input_ids: torch.Tensor, max_new_tokens: int, temperature: float = 0.8, top_k: int = 40,
             top_p: float = 0.9, draft_model=None, speculative_draft_len: int = 0, kvq: str = "none",
             window_size: int = 0, return_stats: bool = False, eos_id: int | None = None, seed: int | None = None,
             max_len: int | None = None, cuda_graph: bool = True, repetition_penalty: float = 1.0,
             presence_penalty: float = 0.0, frequency_penalty: float = 0.0, logit_bias: dict | None = None,
             penalty_window: int = 128,
             # decode-time add-ons (omnicoder.inference.addons)
             knn_cache=None, knn_k: int = 16, knn_lambda: float = 0.2, knn_write_every: int = 8,
             retrieved_texts: list[str] | None = None, retrieval_bias_alpha: float = 0.0, encode_fn=None,
             sfb: bool = False, sfb_alpha: float = 1.0, prompt_text: str | None = None,
             dual_substrate: bool = True, dual_alpha: float = 1.0, dual_beta: float = 1.0,
             adaptive_moe: bool = False, adaptive_top_k_min: int = 1, adaptive_top_k_max: int = 4,
             adaptive_conf_floor: float = 0.3, adaptive_layer_ramp: bool = False, adaptive_layer_power: float = 1.0,
             early_exit: bool = False, early_exit_entropy: float = 0.0, early_exit_mode: str = "entropy",
             verify_threshold: float = 0.0, compress_kv_slots: int = 0, prefix_embeds: torch.Tensor | None = None,
             scmoe_alpha: float = 0.0, scmoe_topk: int = 1, scmoe_frac: float = 1.0, mtp_draft: bool = False):
    """Generate `max_new_tokens` tokens after `input_ids` [B, S] (or [S]).  Returns
    [B, S + max_new_tokens] (and GenStats with return_stats).  On CUDA the
    decode step is captured once as a CUDA graph (`cuda_graph=False` runs it
    eagerly).  Repetition / presence / frequency penalties over the last `penalty_window`
    tokens (0: the whole sequence) and `logit_bias` (LogitProcessor) apply on the plain decode
    path; speculative decoding refuses them (its acceptance test needs the unmodified target
    distribution).

    Add-ons (omnicoder.inference.addons; plain decode path): kNN-LM blend (`knn_cache`,
    `knn_k`, `knn_lambda`), retrieval bias (`retrieved_texts`, `retrieval_bias_alpha`,
    `encode_fn`), structured factor bias (`sfb`, `sfb_alpha`, `prompt_text` or a tokenizer-bound
    `encode_fn`), dual-substrate blend with the model's byte head when it has one, adaptive
    expert count (`adaptive_moe` with the `adaptive_*` knobs; decodes eagerly).  Speculative
    path: `early_exit` skips the draft on confident steps; `verify_threshold` > 0 with a target
    that has a verifier head accepts draft tokens whose verifier probability reaches the
    threshold (the reference's policy) instead of by rejection sampling.
    `compress_kv_slots` sets the number of compressed memory rows; `prefix_embeds` [B, P, D]
    primes the cache with feature vectors before the prompt.

    Self-contrast MoE decoding (`scmoe_alpha` > 0; reference generate.py `--scmoe_alpha / _topk /
    _frac`): a second, weak pass of the same model routes each token to `scmoe_topk` experts in the
    last `scmoe_frac` of the MoE layers (with its own cache), and the step samples from
    (1 + alpha) log p_strong - alpha log p_weak, which favours what the full expert mixture adds
    over the weakened one.  Eager decode (two passes per step)."""
    model.eval()
    squeeze = input_ids.dim() == 1
    ids = input_ids[None] if squeeze else input_ids
    B, S = ids.shape
    dev = ids.device
    cfg = model.cfg
    if window_size:
        cfg.attn.window = window_size
    if compress_kv_slots:
        cfg.attn.mem_slots = int(compress_kv_slots)
    kv_dtype = "int8" if kvq in ("int8", "u8") else "bf16"
    P = 0 if prefix_embeds is None else int(prefix_embeds.shape[1])
    L = max_len or (P + S + max_new_tokens + max(0, speculative_draft_len) + 2)
    gen = None
    if seed is not None:
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
    stats = GenStats(prompt_tokens=B * S)
    from .addons import DecodeAddons, adapt_moe_top_k, clear_moe_top_k, retrieval_vectors, sfb_token_bias
    addons = DecodeAddons(knn_cache=knn_cache, knn_k=knn_k, knn_lambda=knn_lambda, knn_write_every=knn_write_every,
                          dual_alpha=dual_alpha,
                          dual_beta=dual_beta, dual=bool(dual_substrate) and getattr(model, "byte_head", None) is not None)
    if retrieved_texts and retrieval_bias_alpha > 0:
        if encode_fn is None:
            raise ValueError("encode_fn is required when retrieval_bias_alpha > 0 and retrieved_texts are given")
        addons.retrieval_vecs = retrieval_vectors(model, retrieved_texts, encode_fn)
        addons.retrieval_alpha = float(retrieval_bias_alpha)
    if sfb:
        if encode_fn is None:
            raise ValueError("sfb needs encode_fn (and prompt_text, or a tokenizer-bound encode_fn)")
        text = prompt_text
        if text is None:
            tok_obj = getattr(encode_fn, "__self__", None)
            text = tok_obj.decode(ids[0].tolist()) if tok_obj is not None and hasattr(tok_obj, "decode") else ""
        if retrieved_texts:
            text = "\n\n".join(retrieved_texts[:5]) + "\n\n" + text
        addons.sfb_bias = sfb_token_bias(text, encode_fn, cfg.vocab_size, dev)
        addons.sfb_alpha = float(sfb_alpha)
    if scmoe_alpha > 0 and adaptive_moe:
        raise ValueError("scmoe and adaptive_moe both set the routed-expert count: use one")
    if (draft_model is not None or mtp_draft) and speculative_draft_len > 0:
        if repetition_penalty != 1.0 or presence_penalty or frequency_penalty or logit_bias or addons.active \
                or adaptive_moe or scmoe_alpha > 0:
            raise ValueError("speculative decoding samples from the unmodified target distribution: "
                             "penalties, logit_bias and the logit add-ons are not applied there")
        if draft_model is None:
            out = _speculative_mtp(model, ids, max_new_tokens, speculative_draft_len, temperature, top_k, top_p,
                                   kv_dtype, L, gen, stats)
        else:
            out = _speculative(model, draft_model, ids, max_new_tokens, speculative_draft_len, temperature, top_k,
                               top_p, kv_dtype, L, gen, stats, eos_id, early_exit=(early_exit_mode,
                               early_exit_entropy) if early_exit else None, verify_threshold=verify_threshold,
                               prefix_embeds=prefix_embeds)
    else:
        cache = KVCache(cfg, B, L, dev, dtype=model.embed.dtype, kv_dtype=kv_dtype)
        t0 = time.perf_counter()
        if prefix_embeds is not None:
            prime_kv_with_features(model, prefix_embeds.to(dev), cache)
        hidden = None
        if addons.needs_hidden:
            logits, hidden = _prefill(model, ids, cache, return_hidden=True)
        else:
            logits = _prefill(model, ids, cache)
        weak = None
        if scmoe_alpha > 0:
            weak = _WeakRouting(model, scmoe_topk, scmoe_frac, KVCache(cfg, B, L, dev, dtype=model.embed.dtype,
                                                                       kv_dtype=kv_dtype), scmoe_alpha)
            if prefix_embeds is not None:
                with weak:
                    prime_kv_with_features(model, prefix_embeds.to(dev), weak.cache)
            logits = weak.contrast(logits, lambda: _prefill(model, ids, weak.cache))
        if addons.active:
            logits = addons.apply(model, logits, hidden)
        if adaptive_moe:
            adapt_moe_top_k(model, logits, adaptive_top_k_min, adaptive_top_k_max, adaptive_conf_floor,
                            adaptive_layer_ramp, adaptive_layer_power)
        proc = LogitProcessor(B, logits.shape[-1], dev, repetition_penalty, presence_penalty, frequency_penalty,
                              logit_bias, window=penalty_window)
        if proc.active:
            proc.observe(ids)
        tok = sample_next_token(proc(logits), temperature, top_k, top_p, gen)
        if proc.active:
            proc.observe(tok)
        _sync(tok)
        stats.prefill_s = time.perf_counter() - t0
        toks = [tok]
        done = torch.zeros(B, dtype=torch.bool, device=dev)
        step = None
        if cuda_graph and dev.type == "cuda" and max_new_tokens > 2 and not adaptive_moe and weak is None:
            from .graphs import GraphedStep
            step = GraphedStep(model, cache, return_hidden=addons.needs_hidden)
        t1 = time.perf_counter()
        for _ in range(max_new_tokens - 1):
            ts = time.perf_counter()
            if step is not None:
                logits = step(tok[:, None])[:, -1]
                hidden = step.hidden[:, -1] if step.hidden is not None else None
            elif addons.needs_hidden:
                logits, hidden = model.forward_cached(tok[:, None], cache, return_hidden=True)
                logits, hidden = logits[:, -1], hidden[:, -1]
            else:
                logits = model.forward_cached(tok[:, None], cache)[:, -1]
            if weak is not None:
                t_in = tok[:, None]
                logits = weak.contrast(logits, lambda: model.forward_cached(t_in, weak.cache)[:, -1])
            if addons.active:
                logits = addons.apply(model, logits, hidden)
            if adaptive_moe:
                adapt_moe_top_k(model, logits, adaptive_top_k_min, adaptive_top_k_max, adaptive_conf_floor,
                                adaptive_layer_ramp, adaptive_layer_power)
            tok = sample_next_token(proc(logits), temperature, top_k, top_p, gen)
            if proc.active:
                proc.observe(tok)
            if eos_id is not None:
                done |= tok == eos_id
                tok = torch.where(done, torch.full_like(tok, eos_id), tok)
            toks.append(tok)
            stats.steps += 1
            if return_stats:
                _sync(tok)
                stats.step_times_s.append(time.perf_counter() - ts)
        _sync(tok)
        stats.decode_s = time.perf_counter() - t1
        stats.new_tokens = B * (max_new_tokens - 1)
        if adaptive_moe:
            clear_moe_top_k(model)
        out = torch.cat([ids, torch.stack(toks, dim=1)], dim=1)
    out = out[0] if squeeze else out
    return (out, stats) if return_stats else out


class _WeakRouting:
    """The weak pass of self-contrast MoE decoding: `topk` routed experts in the last `frac` of the
    MoE layers while active (context manager), its own KV cache."""

    def __init__(self, model, topk: int, frac: float, cache, alpha: float):
        from ..models.lm import MoEFFN
        moes = [b.ffn for b in model.blocks if isinstance(b.ffn, MoEFFN)]
        n = max(1, int(round(len(moes) * max(0.0, min(1.0, frac))))) if moes else 0
        self.layers, self.topk, self.cache, self.alpha = moes[len(moes) - n:], int(topk), cache, float(alpha)
        self._saved = []

    def __enter__(self):
        self._saved = [m.top_k_override for m in self.layers]
        for m in self.layers:
            m.top_k_override = self.topk
        return self

    def __exit__(self, *exc):
        for m, v in zip(self.layers, self._saved):
            m.top_k_override = v
        return False

    def contrast(self, strong: torch.Tensor, weak_fn) -> torch.Tensor:
        with self:
            weak = weak_fn()
        return ((1 + self.alpha) * torch.log_softmax(strong.float(), -1)
                - self.alpha * torch.log_softmax(weak.float(), -1)).to(strong.dtype)


def _speculative(target, draft, ids, max_new, k, temperature, top_k, top_p, kv_dtype, L, gen, stats, eos_id,
                 early_exit=None, verify_threshold: float = 0.0, prefix_embeds=None):
    """Draft proposes k tokens autoregressively; the target scores all k+1 positions
    in one forward; tokens are accepted left to right with probability
    min(1, p_target/p_draft) (always, when greedy and equal); the first rejection
    is replaced by a sample from normalize(max(0, p_target - p_draft)) and, if all
    k are accepted, a bonus token comes from the target's last position.  Both
    caches are then rolled back per sequence to the accepted length; every sequence
    keeps its own accepted length.

    verify_threshold > 0 with a target that has a verifier head: a draft token is accepted
    while the verifier's probability of it reaches the threshold (reference
    src/omnicoder/inference/generate.py:2925-3048); the next token then comes from the
    target distribution at the first unaccepted position.
    early_exit = (mode, threshold): after a confident step (omnicoder.inference.addons.confident)
    the next step is a single target step without a draft (reference :2433-2467)."""
    from ..ops.spec import spec_verify
    from .addons import confident
    B, S = ids.shape
    dev = ids.device
    # unfiltered sampling (or greedy) verifies in the fused kernel (omnicoder/csrc/spec_verify.cu)
    fused_verify = (not (verify_threshold > 0 and getattr(target, "verifier", None) is not None)
                    and (temperature <= 0 or ((not top_k or top_k <= 0) and (top_p is None or top_p >= 1.0))))
    tcache = KVCache(target.cfg, B, L, dev, dtype=target.embed.dtype, kv_dtype=kv_dtype)
    dcache = KVCache(draft.cfg, B, L, dev, dtype=draft.embed.dtype, kv_dtype="bf16")
    use_verifier = verify_threshold > 0 and getattr(target, "verifier", None) is not None
    t0 = time.perf_counter()
    if prefix_embeds is not None:                   # the draft has another width: only the target is primed
        prime_kv_with_features(target, prefix_embeds.to(dev), tcache)
    if S > 1:
        target.forward_cached(ids[:, :-1], tcache, prefill=True, last_only=True)
        draft.forward_cached(ids[:, :-1], dcache, prefill=True, last_only=True)
    last = ids[:, -1]
    _sync(last)
    stats.prefill_s = time.perf_counter() - t0
    produced = [[] for _ in range(B)]
    t1 = time.perf_counter()
    ar = torch.arange(B, device=dev)
    skip_draft = False
    def keep(base, grown):
        """Sequences that already have max_new tokens stop advancing their cache: while slower
        sequences catch up, their (ignored) writes stay within the last k + 1 rows."""
        done = torch.tensor([len(p) >= max_new for p in produced], device=dev)
        return torch.where(done, base, grown.to(base.dtype))

    while min(len(p) for p in produced) < max_new:
        ts = time.perf_counter()
        if skip_draft:
            # early exit: one target step, the draft cache follows with the same token
            base_t, base_d = tcache.lengths.clone(), dcache.lengths.clone()
            tl = target.forward_cached(last[:, None], tcache)[:, -1]
            draft.forward_cached(last[:, None], dcache)
            tcache.rollback(keep(base_t, tcache.lengths))
            dcache.rollback(keep(base_d, dcache.lengths))
            pt = sampling_probs(tl, temperature, top_k, top_p)
            extra = pt.argmax(-1) if temperature <= 0 else torch.multinomial(pt, 1, generator=gen).squeeze(1)
            for b, e in enumerate(extra.tolist()):
                if len(produced[b]) < max_new:
                    produced[b].append(e)
            stats.steps += 1
            stats.early_exits += 1
            skip_draft = confident(tl, *early_exit)
            last = extra
            _sync(last)
            stats.step_times_s.append(time.perf_counter() - ts)
            continue
        base_t = tcache.lengths.clone()
        base_d = dcache.lengths.clone()
        cur = last
        d_tok, d_prob = [], []
        for _ in range(k):
            dl = draft.forward_cached(cur[:, None], dcache)[:, -1]
            pd = sampling_probs(dl, temperature, top_k, top_p)
            nxt = pd.argmax(-1) if temperature <= 0 else torch.multinomial(pd, 1, generator=gen).squeeze(1)
            d_tok.append(nxt)
            d_prob.append(pd)
            cur = nxt
        d_tok_t = torch.stack(d_tok, dim=1)                          # [B, k]
        seq_in = torch.cat([last[:, None], d_tok_t], dim=1)
        if use_verifier:
            tl, th = target.forward_cached(seq_in, tcache, return_hidden=True)      # [B, k+1, V], [B, k+1, D]
        else:
            tl = target.forward_cached(seq_in, tcache)
        pd_all = torch.stack(d_prob, dim=1)                          # [B, k, V]
        if fused_verify:
            # one kernel: per-sequence acceptance, next token and rolled-back cache lengths
            u = torch.rand(B, k + 1, device=dev, generator=gen) if temperature > 0 else None
            n_acc, extra, new_len = spec_verify(tl, pd_all if temperature > 0 else None, d_tok_t, u, base_t,
                                                temperature)
            draft.forward_cached(d_tok_t[:, -1:], dcache)
            tcache.rollback(keep(base_t, new_len))
            dcache.rollback(keep(base_d, base_d + (n_acc + 1).to(base_d.dtype)))
            n_list, d_list, e_list = n_acc.tolist(), d_tok_t.tolist(), extra.tolist()
            for b in range(B):
                if len(produced[b]) < max_new:
                    produced[b].extend(d_list[b][:n_list[b]] + [e_list[b]])
            stats.accepted_draft_tokens += int(sum(n_list))
            stats.proposed_draft_tokens += B * k
            stats.steps += 1
            if early_exit is not None:
                skip_draft = confident(tl[ar, n_acc.long()], *early_exit)
            last = extra
            _sync(last)
            stats.step_times_s.append(time.perf_counter() - ts)
            continue
        pt = sampling_probs(tl, temperature, top_k, top_p)           # [B, k+1, V]
        if use_verifier:
            vl = (th[:, :k].to(target.verifier.dtype) @ target.verifier.t()).float()
            v_d = torch.softmax(vl, -1).gather(-1, d_tok_t[..., None]).squeeze(-1)
            acc = v_d >= verify_threshold
        else:
            pt_d = pt[:, :k].gather(-1, d_tok_t[..., None]).squeeze(-1)
            pd_d = pd_all.gather(-1, d_tok_t[..., None]).squeeze(-1)
            if temperature <= 0:
                acc = pt_d > 0.5
            else:
                u = torch.rand(B, k, device=dev, generator=gen)
                acc = u < torch.clamp(pt_d / pd_d.clamp_min(1e-20), max=1.0)
        n_acc = torch.cumprod(acc.int(), dim=1).sum(1)               # accepted prefix length [B]
        # correction / bonus token at position n_acc
        p_next = pt[ar, n_acc]                                       # [B, V]
        if use_verifier:
            q = p_next
        else:
            resid = torch.clamp(p_next - torch.cat([pd_all, torch.zeros_like(pd_all[:, :1])], 1)[ar, n_acc], min=0)
            q = torch.where((n_acc < k)[:, None], resid, p_next)
        q = q / q.sum(-1, keepdim=True).clamp_min(1e-20)
        extra = q.argmax(-1) if temperature <= 0 else torch.multinomial(q, 1, generator=gen).squeeze(1)
        # draft cache lacks the k-th draft token when everything was accepted: catch up
        draft.forward_cached(d_tok_t[:, -1:], dcache)
        tcache.rollback(keep(base_t, base_t + n_acc + 1))
        dcache.rollback(keep(base_d, base_d + n_acc + 1))
        n_list = n_acc.tolist()
        d_list = d_tok_t.tolist()
        e_list = extra.tolist()
        for b in range(B):
            if len(produced[b]) < max_new:
                produced[b].extend(d_list[b][:n_list[b]] + [e_list[b]])
        stats.accepted_draft_tokens += int(sum(n_list))
        stats.proposed_draft_tokens += B * k
        stats.steps += 1
        if early_exit is not None:
            skip_draft = confident(tl[ar, n_acc], *early_exit)
        last = extra
        _sync(last)
        stats.step_times_s.append(time.perf_counter() - ts)
    stats.decode_s = time.perf_counter() - t1
    stats.new_tokens = B * max_new
    out = torch.tensor([p[:max_new] for p in produced], device=dev, dtype=ids.dtype)
    return torch.cat([ids, out], dim=1)


def _speculative_mtp(target, ids, max_new, k, temperature, top_k, top_p, kv_dtype, L, gen, stats):
    """Self-speculative decoding from the target's multi-token-prediction heads (the reference's
    --multi_token_heads lookahead, src/omnicoder/inference/generate.py:3970).  The final hidden state h
    at the position that produced `last` gives, through MTP head j, a proposal for the token j + 1
    places after `last` (the heads are trained that way: head j at position t predicts token
    t + 2 + j).  The k proposals (k <= number of MTP heads) are verified with one target forward of
    [last, d_1 .. d_k] exactly as a draft model's would be (rejection sampling, or equality when
    greedy), and the hidden state at the position that produced the next token feeds the next round's
    proposals; the cache is rolled back per sequence to the accepted length."""
    from ..ops.layers import linear
    from ..ops.spec import spec_verify
    heads = list(target.mtp_heads)
    if not heads:
        raise ValueError("self-speculative decoding needs a model with MTP heads (cfg.mtp_heads > 0)")
    k = min(k, len(heads))
    B, S = ids.shape
    dev = ids.device
    tcache = KVCache(target.cfg, B, L, dev, dtype=target.embed.dtype, kv_dtype=kv_dtype)
    t0 = time.perf_counter()
    produced = [[] for _ in range(B)]
    if S > 1:
        _, h = target.forward_cached(ids[:, :-1], tcache, prefill=True, last_only=True, return_hidden=True)
        h = h[:, -1]
        last = ids[:, -1]
    else:                                             # no prompt context yet: one plain step first
        tl, h = target.forward_cached(ids, tcache, prefill=True, last_only=True, return_hidden=True)
        pt = sampling_probs(tl[:, -1], temperature, top_k, top_p)
        last = pt.argmax(-1) if temperature <= 0 else torch.multinomial(pt, 1, generator=gen).squeeze(1)
        h = h[:, -1]
        for b, e in enumerate(last.tolist()):
            produced[b].append(e)
    _sync(last)
    stats.prefill_s = time.perf_counter() - t0
    t1 = time.perf_counter()
    ar = torch.arange(B, device=dev)
    while min(len(p) for p in produced) < max_new:
        ts = time.perf_counter()
        base_t = tcache.lengths.clone()
        d_tok, d_prob = [], []
        for j in range(k):
            pd = sampling_probs(linear(h, heads[j]).float(), temperature, top_k, top_p)
            d_tok.append(pd.argmax(-1) if temperature <= 0 else torch.multinomial(pd, 1, generator=gen).squeeze(1))
            d_prob.append(pd)
        d_tok_t = torch.stack(d_tok, dim=1)                                  # [B, k]
        pd_all = torch.stack(d_prob, dim=1)                                  # [B, k, V]
        tl, th = target.forward_cached(torch.cat([last[:, None], d_tok_t], 1), tcache, return_hidden=True)
        if temperature <= 0 or ((not top_k or top_k <= 0) and (top_p is None or top_p >= 1.0)):
            u = torch.rand(B, k + 1, device=dev, generator=gen) if temperature > 0 else None
            n_acc, extra, new_len = spec_verify(tl, pd_all if temperature > 0 else None, d_tok_t, u, base_t,
                                                temperature)
        else:
            pt = sampling_probs(tl, temperature, top_k, top_p)
            pt_d = pt[:, :k].gather(-1, d_tok_t[..., None]).squeeze(-1)
            pd_d = pd_all.gather(-1, d_tok_t[..., None]).squeeze(-1)
            acc = torch.rand(B, k, device=dev, generator=gen) < torch.clamp(pt_d / pd_d.clamp_min(1e-20), max=1.0)
            n_acc = torch.cumprod(acc.int(), dim=1).sum(1)
            p_next = pt[ar, n_acc]
            resid = torch.clamp(p_next - torch.cat([pd_all, torch.zeros_like(pd_all[:, :1])], 1)[ar, n_acc], min=0)
            q = torch.where((n_acc < k)[:, None], resid, p_next)
            q = q / q.sum(-1, keepdim=True).clamp_min(1e-20)
            extra = torch.multinomial(q, 1, generator=gen).squeeze(1)
            new_len = base_t + n_acc + 1
        done = torch.tensor([len(p) >= max_new for p in produced], device=dev)
        tcache.rollback(torch.where(done, base_t, new_len.to(base_t.dtype)))
        n_list, d_list, e_list = n_acc.tolist(), d_tok_t.tolist(), extra.tolist()
        for b in range(B):
            if len(produced[b]) < max_new:
                produced[b].extend(d_list[b][:n_list[b]] + [e_list[b]])
        stats.accepted_draft_tokens += int(sum(n_list))
        stats.proposed_draft_tokens += B * k
        stats.steps += 1
        h = th[ar, n_acc.long()]                    # the hidden state that produced `extra`
        last = extra
        _sync(last)
        stats.step_times_s.append(time.perf_counter() - ts)
    stats.decode_s = time.perf_counter() - t1
    stats.new_tokens = B * max_new
    out = torch.tensor([p[:max_new] for p in produced], device=dev, dtype=ids.dtype)
    return torch.cat([ids, out], dim=1)


# ----------------------------------------------------------------------------
# CLI (python -m omnicoder.inference.generate)
# ----------------------------------------------------------------------------
def main(argv=None):
    from ..config import get_preset
    from ..models.lm import build_model
    from ..training.checkpoint import maybe_load_checkpoint
    from ..training.tokenizer import get_tokenizer

    ap = argparse.ArgumentParser(description="omnicoder text generation")
    ap.add_argument("--prompt", default="def fibonacci(n):")
    ap.add_argument("--preset", default="tiny_moe")
    ap.add_argument("--ckpt", default=None)
    ap.add_argument("--max_new_tokens", type=int, default=64)
    ap.add_argument("--temperature", type=float, default=0.8)
    ap.add_argument("--top_k", type=int, default=40)
    ap.add_argument("--top_p", type=float, default=0.9)
    ap.add_argument("--repetition_penalty", type=float, default=1.0)
    ap.add_argument("--presence_penalty", type=float, default=0.0)
    ap.add_argument("--frequency_penalty", type=float, default=0.0)
    ap.add_argument("--logit_bias_file", default=None, help="JSON {token id: additive bias}")
    ap.add_argument("--kvq", default="none", choices=["none", "int8", "u8"])
    ap.add_argument("--window_size", type=int, default=0)
    ap.add_argument("--draft_preset", default=None)
    ap.add_argument("--draft_ckpt", default=None)
    ap.add_argument("--speculative_draft_len", type=int, default=0)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--penalty_window", type=int, default=128, help="tokens the penalties look back over (0: all)")
    ap.add_argument("--eos_id", type=int, default=None)
    ap.add_argument("--no_cuda_graph", action="store_true", help="decode eagerly instead of replaying a CUDA graph")
    # add-ons
    ap.add_argument("--knn_cache", default=None, help="saved kNN-LM cache (KNNCache.save) to blend with")
    ap.add_argument("--knn_k", type=int, default=16)
    ap.add_argument("--knn_lambda", type=float, default=0.2)
    ap.add_argument("--retrieve_texts", default=None, help="file with one retrieved passage per line")
    ap.add_argument("--retrieval_bias_alpha", type=float, default=0.0)
    ap.add_argument("--sfb", action="store_true", help="structured factor bias from the factorised prompt")
    ap.add_argument("--sfb_alpha", type=float, default=1.0)
    ap.add_argument("--adaptive_moe", "--adaptive_gating", dest="adaptive_moe", action="store_true",
                    help="confidence-driven routed experts per token")
    ap.add_argument("--adaptive_top_k_min", type=int, default=1)
    ap.add_argument("--adaptive_top_k_max", type=int, default=4)
    ap.add_argument("--adaptive_conf_floor", type=float, default=0.3)
    ap.add_argument("--adaptive_layer_ramp", action="store_true")
    ap.add_argument("--early_exit", action="store_true", help="skip the speculative draft on confident steps")
    ap.add_argument("--early_exit_entropy", type=float, default=1.0)
    ap.add_argument("--early_exit_mode", default="entropy", choices=["entropy", "delta"])
    ap.add_argument("--verify_threshold", type=float, default=0.0,
                    help="speculative acceptance by the target's verifier head (0: rejection sampling)")
    ap.add_argument("--compress_kv_slots", type=int, default=0, help="compressed memory rows of the cache")
    ap.add_argument("--mem_slots", type=int, default=None, help="alias of --compress_kv_slots")
    ap.add_argument("--scmoe_alpha", type=float, default=0.0, help="self-contrast MoE strength (0: off)")
    ap.add_argument("--scmoe_topk", type=int, default=1, help="routed experts of the weak pass")
    ap.add_argument("--scmoe_frac", type=float, default=1.0, help="fraction of (last) MoE layers weakened")
    ap.add_argument("--adaptive_layer_power", type=float, default=1.0)
    # model / context
    ap.add_argument("--mobile_preset", default=None, help="alias of --preset")
    ap.add_argument("--rope_scale", type=float, default=None, help="divide RoPE positions by this factor")
    ap.add_argument("--rope_base", type=float, default=None, help="RoPE base (theta)")
    ap.add_argument("--target_ctx", type=int, default=0,
                    help="extend the context to this length (RoPE position interpolation)")
    ap.add_argument("--disable_speculative", action="store_true")
    ap.add_argument("--reasoner", default="none", choices=["none", "tot", "omega"],
                    help="tot: a tree-of-thoughts MCTS over the next tokens picks the opening of the answer; "
                         "omega: attach the verification certificate (as --emit_cert)")
    ap.add_argument("--tree_depth", type=int, default=3, help="tokens chosen by the tree search")
    ap.add_argument("--tree_width", type=int, default=3, help="next tokens expanded per node")
    ap.add_argument("--tree_iterations", type=int, default=24)
    ap.add_argument("--multi_token_heads", type=int, default=0,
                    help="build the model with this many prediction heads (main + MTP); with > 1 and no draft "
                         "model, decoding drafts from the MTP heads (self-speculative)")
    # prompt
    ap.add_argument("--system_prompt", default="")
    ap.add_argument("--prompt_template", default="{system}{prompt}",
                    help="format string with {system} and {prompt}")
    # retrieval from local files
    ap.add_argument("--retrieve_path", default=None, help="folder (or file) of .txt / .md / .py documents")
    ap.add_argument("--retrieve_k", type=int, default=3)
    ap.add_argument("--retrieve_chunk", type=int, default=600, help="characters per chunk")
    ap.add_argument("--retrieve_stride", type=int, default=400)
    ap.add_argument("--retrieve_max_chars", type=int, default=2000, help="retrieved characters put in the prompt")
    ap.add_argument("--retrieve_prepend", action="store_true", help="put the retrieved passages before the prompt")
    ap.add_argument("--pref_lora", default=None, help="preference-expert LoRA adapters to load onto the model")
    ap.add_argument("--pref_index", "--pref_rag_index", dest="pref_index", default=None,
                    help="preference-expert retrieval index (a saved PQ index)")
    ap.add_argument("--pref_k", "--pref_rag_topk", dest="pref_k", type=int, default=2,
                    help="passages taken from --pref_index")
    ap.add_argument("--pref_rag_alpha", type=float, default=None,
                    help="retrieval-bias strength of the preference passages (sets --retrieval_bias_alpha)")
    ap.add_argument("--pref_lora_r", type=int, default=None, help="expected adapter rank (checked against the file)")
    ap.add_argument("--pref_lora_alpha", type=int, default=None, help="expected adapter alpha (checked)")
    ap.add_argument("--pref_lora_dropout", type=float, default=0.0, help="accepted; adapters run without dropout")
    ap.add_argument("--retrieve_pq_index", default=None, help="a saved PQ index (pq-build) to retrieve from")
    ap.add_argument("--multi_index_root", default=None,
                    help="folder of saved PQ indexes: each is searched and the best passages merged")
    ap.add_argument("--mi_topk", type=int, default=3, help="passages kept from --multi_index_root")
    ap.add_argument("--mi_alpha", type=float, default=None,
                    help="retrieval-bias strength of the multi-index passages (sets --retrieval_bias_alpha)")
    ap.add_argument("--retrieve_budget_bytes", type=int, default=0,
                    help="cap the retrieved passages at this many UTF-8 bytes (0: no cap)")
    ap.add_argument("--retrieve_faiss", default=None, help="not available: FAISS is not installed (use pq-build)")
    ap.add_argument("--retrieve_partition", default=None, help="not available (use --multi_index_root)")
    ap.add_argument("--compile", action="store_true", help="not used: decode steps replay CUDA graphs instead")
    # post-processing
    ap.add_argument("--tool_use", action="store_true", help="run <tool>name(args)</tool> calls in the output")
    ap.add_argument("--emit_cert", action="store_true", help="print a proof-carrying answer record (JSON)")
    ap.add_argument("--proof_margin_thresh", type=float, default=0.0,
                    help="with --emit_cert: abstain when the verification margin is below this")
    a = ap.parse_args(argv)
    cfg = get_preset(a.mobile_preset or a.preset)
    if a.multi_token_heads > 1:
        cfg.mtp_heads = a.multi_token_heads - 1
    if a.rope_scale is not None:
        cfg.attn.rope_scale = a.rope_scale
    if a.rope_base is not None:
        cfg.attn.rope_theta = a.rope_base
    if a.target_ctx:
        from ..config import get_rope_scale_for_target_ctx
        cfg.attn.rope_scale *= get_rope_scale_for_target_ctx(cfg.max_seq_len, a.target_ctx)
        cfg.max_seq_len = max(cfg.max_seq_len, a.target_ctx)
    if a.mem_slots is not None:
        a.compress_kv_slots = a.mem_slots
    if a.disable_speculative:
        a.draft_preset, a.speculative_draft_len = None, 0
    model = build_model(cfg, device=a.device)
    if a.ckpt:
        maybe_load_checkpoint(model, a.ckpt)
    for flag in ("retrieve_faiss", "retrieve_partition"):
        if getattr(a, flag):
            raise SystemExit(f"--{flag} is not available here: FAISS is not installed; build a PQ index with "
                             f"`python -m omnicoder.tools.utilities pq-build` and pass --retrieve_pq_index")
    if a.compile:
        print("[generate] --compile has no effect: decode steps are captured as CUDA graphs", file=sys.stderr)
    if a.pref_lora:
        from ..training.preference_expert import load_preference_lora
        if a.pref_lora_r is not None or a.pref_lora_alpha is not None:
            meta = torch.load(a.pref_lora, map_location="cpu", weights_only=True)
            for key, want in (("r", a.pref_lora_r), ("alpha", a.pref_lora_alpha)):
                if want is not None and int(meta[key]) != want:
                    raise SystemExit(f"--pref_lora_{key} {want} does not match the adapters ({meta[key]})")
        load_preference_lora(model, a.pref_lora)
    for alpha in (a.pref_rag_alpha, a.mi_alpha):
        if alpha is not None:
            a.retrieval_bias_alpha = alpha
    tok = get_tokenizer(cfg.vocab_size)
    passages = []
    if a.retrieve_path:
        passages = retrieve_passages(a.retrieve_path, a.prompt, a.retrieve_k, a.retrieve_chunk, a.retrieve_stride)
    if a.pref_index or a.retrieve_pq_index or a.multi_index_root:
        from ..retrieval.pq import PQRetriever
        if a.pref_index:
            passages += [d for _, _, d in PQRetriever.load(a.pref_index).search(a.prompt, a.pref_k)]
        if a.retrieve_pq_index:
            passages += [d for _, _, d in PQRetriever.load(a.retrieve_pq_index).search(a.prompt, a.retrieve_k)]
        if a.multi_index_root:
            import os
            hits = []
            for d in sorted(os.listdir(a.multi_index_root)):
                sub = os.path.join(a.multi_index_root, d)
                if os.path.exists(os.path.join(sub, "pq.json")):
                    # distances of different indexes are comparable: unit-norm vectors in each
                    hits += [(dist, doc) for _, dist, doc in PQRetriever.load(sub).search(a.prompt, a.mi_topk)]
            passages += [doc for _, doc in sorted(hits, key=lambda t: t[0])[:a.mi_topk]]
    if a.retrieve_budget_bytes > 0:
        kept, used = [], 0
        for ptxt in passages:
            b = len(ptxt.encode("utf-8"))
            if used + b > a.retrieve_budget_bytes:
                break
            kept.append(ptxt)
            used += b
        passages = kept
    context = ""
    if a.retrieve_prepend and passages:
        context = "\n".join(passages)[:a.retrieve_max_chars] + "\n"
    prompt_text = context + a.prompt_template.format(system=a.system_prompt, prompt=a.prompt)
    ids = torch.tensor([tok.encode(prompt_text)], device=a.device)
    if a.reasoner == "omega":
        a.emit_cert = True
    tree_ids = []
    if a.reasoner == "tot" and a.tree_depth > 0:
        from ..reasoning.lm_search import LMToTMCTS, ToTConfig
        search = LMToTMCTS(model.eval(), tok, ToTConfig(branch=a.tree_width, max_depth=a.tree_depth,
                                                        iterations=a.tree_iterations))
        tree_ids, _ = search.search(prompt_text)
        ids = torch.cat([ids, torch.tensor([tree_ids], device=a.device, dtype=ids.dtype)], 1)
        a.max_new_tokens = max(1, a.max_new_tokens - len(tree_ids))
    draft = None
    if a.draft_preset:
        draft = build_model(get_preset(a.draft_preset), device=a.device)
        if a.draft_ckpt:
            maybe_load_checkpoint(draft, a.draft_ckpt)
    knn = None
    if a.knn_cache:
        from .knn_cache import KNNCache
        knn = KNNCache.load(a.knn_cache)
    texts = None
    if a.retrieve_texts:
        with open(a.retrieve_texts) as f:
            texts = [ln.strip() for ln in f if ln.strip()]
    if passages:
        texts = (texts or []) + passages
    out, st = generate(model, ids, a.max_new_tokens, a.temperature, a.top_k, a.top_p, draft_model=draft,
                       repetition_penalty=a.repetition_penalty, presence_penalty=a.presence_penalty,
                       frequency_penalty=a.frequency_penalty,
                       logit_bias=load_logit_bias(a.logit_bias_file) if a.logit_bias_file else None,
                       speculative_draft_len=(a.speculative_draft_len or max(0, a.multi_token_heads - 1))
                       if not a.disable_speculative else 0,
                       mtp_draft=a.multi_token_heads > 1 and draft is None, kvq=a.kvq, window_size=a.window_size,
                       return_stats=True, seed=a.seed, eos_id=a.eos_id, cuda_graph=not a.no_cuda_graph,
                       penalty_window=a.penalty_window, knn_cache=knn, knn_k=a.knn_k, knn_lambda=a.knn_lambda,
                       retrieved_texts=texts, retrieval_bias_alpha=a.retrieval_bias_alpha, encode_fn=tok.encode,
                       sfb=a.sfb, sfb_alpha=a.sfb_alpha, prompt_text=a.prompt, adaptive_moe=a.adaptive_moe,
                       adaptive_top_k_min=a.adaptive_top_k_min, adaptive_top_k_max=a.adaptive_top_k_max,
                       adaptive_conf_floor=a.adaptive_conf_floor, adaptive_layer_ramp=a.adaptive_layer_ramp,
                       early_exit=a.early_exit, early_exit_entropy=a.early_exit_entropy,
                       early_exit_mode=a.early_exit_mode, verify_threshold=a.verify_threshold,
                       compress_kv_slots=a.compress_kv_slots, adaptive_layer_power=a.adaptive_layer_power,
                       scmoe_alpha=a.scmoe_alpha, scmoe_topk=a.scmoe_topk, scmoe_frac=a.scmoe_frac)
    text = tok.decode(tree_ids + out[0, ids.shape[1]:].tolist())
    if a.tool_use:
        from .tools import ToolRegistry
        text = ToolRegistry().run_calls(text)
    result = {"text": text, "stats": st.as_dict(), "retrieved_passages": len(passages)}
    if a.emit_cert:
        from ..reasoning.omega import infer_goals, pack_certificate, text_margin
        cert = pack_certificate(text, infer_goals(a.prompt), {"text": text_margin(text, " ".join(passages) or None)})
        result["certificate"] = json.loads(cert.to_json())
        if cert.margin < a.proof_margin_thresh:
            result["abstained"] = True
            text = ""
    if a.json:
        print(json.dumps(result))
    else:
        print(text)
        print(json.dumps({k: v for k, v in result.items() if k != "text"}), file=sys.stderr)


def retrieve_passages(path: str, query: str, k: int = 3, chunk: int = 600, stride: int = 400) -> list[str]:
    """Top-k chunks of the documents under `path` for `query` (character windows of `chunk` with
    step `stride`, ranked by the TF-IDF product-quantisation retriever)."""
    import os

    from ..retrieval.pq import PQRetriever
    files = [path] if os.path.isfile(path) else [
        os.path.join(r, f) for r, _, fs in os.walk(path) for f in sorted(fs) if f.endswith((".txt", ".md", ".py"))]
    docs = []
    for fp in sorted(files):
        with open(fp, encoding="utf-8", errors="ignore") as f:
            t = f.read()
        docs += [t[i:i + chunk] for i in range(0, max(1, len(t) - chunk + stride), max(1, stride)) if t[i:i + chunk].strip()]
    if not docs:
        return []
    r = PQRetriever(n_subspaces=4, n_centroids=min(16, len(docs))).fit(docs)
    return [d for _, _, d in r.search(query, k)]


if __name__ == "__main__":
    main()
