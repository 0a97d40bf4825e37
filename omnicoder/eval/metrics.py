"""Evaluation metrics (reference src/omnicoder/eval/*: auto_benchmark, text/code evals).

* perplexity over token windows (mean CE exponentiated);
* evaluate_qa: greedy answers scored by exact or numeric match;
* pass_at_k: the unbiased estimator 1 - C(n - c, k) / C(n, k) (Chen et al. 2021,
  "Evaluating Large Language Models Trained on Code");
* evaluate_code: n samples per task, tests run in the sandbox of
  omnicoder.training.rl, pass@k averaged over tasks;
* auto_benchmark: perplexity + generation throughput in one JSON-able dict.
"""
from __future__ import annotations

import math

import torch

from ..inference.generate import generate


@torch.no_grad()
def perplexity(model, windows: list[torch.Tensor]) -> float:
    """windows: token id tensors [S + 1]; returns exp(mean CE)."""
    tot, n = 0.0, 0
    dev = next(model.parameters()).device
    for w in windows:
        w = w.to(dev)
        out = model(w[None, :-1], labels=w[None, 1:])
        tot += float(out["ce"]) * (w.numel() - 1)
        n += w.numel() - 1
    return math.exp(tot / max(1, n))


def pass_at_k(n: int, c: int, k: int) -> float:
    if n - c < k:
        return 1.0
    return 1.0 - math.prod((n - c - i) / (n - i) for i in range(k))


@torch.no_grad()
def evaluate_qa(model, tokenizer, items: list[dict], max_new_tokens: int = 32, numeric: bool = False) -> dict:
    from ..training.rl import reward_exact, reward_numeric
    dev = next(model.parameters()).device
    score = 0.0
    for it in items:
        ids = torch.tensor([tokenizer.encode(it["question"])], device=dev)
        out = generate(model, ids, max_new_tokens, temperature=0.0)
        pred = tokenizer.decode(out[0, ids.shape[1]:].tolist())
        score += (reward_numeric if numeric else reward_exact)(pred, it["answer"])
    return {"accuracy": score / max(1, len(items)), "n": len(items)}


@torch.no_grad()
def evaluate_code(model, tokenizer, tasks: list[dict], n: int = 4, k: int = 1, max_new_tokens: int = 128,
                  temperature: float = 0.8, timeout_s: float = 5.0) -> dict:
    """tasks: {"prompt": str, "tests": [assert statements]}."""
    from ..training.rl import reward_code
    dev = next(model.parameters()).device
    vals = []
    for t in tasks:
        ids = torch.tensor([tokenizer.encode(t["prompt"])], device=dev).repeat(n, 1)
        outs = generate(model, ids, max_new_tokens, temperature=temperature, top_k=0, top_p=0.95, seed=0)
        c = sum(reward_code(t["prompt"] + tokenizer.decode(o[ids.shape[1]:].tolist()), t["tests"], timeout_s) == 1.0
                for o in outs)
        vals.append(pass_at_k(n, c, k))
    return {f"pass@{k}": sum(vals) / max(1, len(vals)), "tasks": len(tasks)}


def auto_benchmark(model, windows: list[torch.Tensor] | None = None, seq_len: int = 64, gen_tokens: int = 32,
                   batch: int = 4) -> dict:
    from ..inference.benchmark import decode_benchmark
    out = decode_benchmark(model, batch, seq_len, gen_tokens)
    if windows:
        out["perplexity"] = perplexity(model, windows)
    return out
