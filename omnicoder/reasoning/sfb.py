"""Structured factor blending (reference src/omnicoder/sfb/: factorize.py:1-454,
factor solvers, compile/spn.py:1-337, fusion/cross_bias.py:1-168,
arbiter.py:1-247).

factorize(prompt): splits a request into typed sub-goals (numbered / bulleted
items, "and"-joined clauses, question sentences), each tagged math / code /
retrieval / text by keyword rules.
SumProductNetwork: leaf indicator distributions, product and weighted sum
nodes; `value(evidence)` evaluates bottom-up, `marginal(var)` by evaluating
with each value of the variable clamped (the compiled form of a small
factor graph: `compile_factor_graph` enumerates the joint of discrete
factors into a sum over products).
cross_bias: fuses per-factor token preferences into one additive logit bias
(log of a weighted mixture of the factors' distributions).
ProofMarginArbiter: picks among candidate answers by (verified, margin between
the best and second-best scores), abstaining when the margin is below a threshold.
"""
from __future__ import annotations

import itertools
import math
import re

import torch

_KINDS = [("math", r"\b(compute|calculate|sum|integral|solve|equation|\d+\s*[-+*/^]\s*\d+)"),
          ("code", r"\b(code|function|python|implement|bug|compile|class)\b"),
          ("retrieval", r"\b(who|when|where|cite|source|according)\b")]


def factorize(prompt: str) -> list[dict]:
    parts = re.split(r"(?:^|\n)\s*(?:\d+[.)]|[-*])\s+", prompt)
    parts = [p.strip() for p in parts if p.strip()]
    if len(parts) <= 1:
        parts = [p.strip() for p in re.split(r"(?<=[?.!])\s+|\band then\b|;\s*", prompt) if p.strip()]
    out = []
    for p in parts:
        kind = "text"
        for k, rx in _KINDS:
            if re.search(rx, p, re.I):
                kind = k
                break
        out.append({"goal": p, "kind": kind})
    return out


class SumProductNetwork:
    """Nodes: ("leaf", var, value) indicator, ("prod", [children]), ("sum", [(weight, child)])."""

    def __init__(self, root):
        self.root = root

    def _eval(self, node, ev: dict) -> float:
        t = node[0]
        if t == "leaf":
            _, var, val = node
            return 1.0 if ev.get(var, val) == val else 0.0
        if t == "prod":
            r = 1.0
            for c in node[1]:
                r *= self._eval(c, ev)
            return r
        return sum(w * self._eval(c, ev) for w, c in node[1])

    def value(self, evidence: dict | None = None) -> float:
        return self._eval(self.root, evidence or {})

    def marginal(self, var: str, values, evidence: dict | None = None) -> dict:
        ev = dict(evidence or {})
        z = self.value(ev)
        out = {}
        for v in values:
            ev[var] = v
            out[v] = self.value(ev) / z if z > 0 else 0.0
        return out


def compile_factor_graph(variables: dict, factors: list) -> SumProductNetwork:
    """variables: name -> list of values; factors: (vars tuple, fn(*values) -> weight >= 0).
    The network is a weighted sum over every joint assignment of a product of indicators."""
    names = list(variables)
    terms = []
    for assign in itertools.product(*[variables[n] for n in names]):
        a = dict(zip(names, assign))
        w = 1.0
        for vs, fn in factors:
            w *= fn(*[a[v] for v in vs])
        if w > 0:
            terms.append((w, ("prod", [("leaf", n, a[n]) for n in names])))
    return SumProductNetwork(("sum", terms))


def cross_bias(factor_probs: list[torch.Tensor], weights: list[float] | None = None, strength: float = 1.0,
               eps: float = 1e-8) -> torch.Tensor:
    """log(sum_i w_i p_i) - log(uniform), scaled: an additive logit bias from per-factor distributions."""
    w = torch.tensor(weights if weights is not None else [1.0] * len(factor_probs))
    w = w / w.sum()
    mix = sum(wi * p for wi, p in zip(w.tolist(), factor_probs))
    V = mix.shape[-1]
    return strength * (torch.log(mix + eps) + math.log(V))


class ProofMarginArbiter:
    def __init__(self, margin: float = 0.1):
        self.margin = margin

    def choose(self, candidates: list[dict]):
        """candidates: {"answer", "score", "verified": bool}; verified answers win; returns the
        answer or None (abstain) when the top two are within the margin."""
        if not candidates:
            return None
        ranked = sorted(candidates, key=lambda c: (bool(c.get("verified")), c["score"]), reverse=True)
        if len(ranked) > 1 and bool(ranked[0].get("verified")) == bool(ranked[1].get("verified")) and \
                ranked[0]["score"] - ranked[1]["score"] < self.margin:
            return None
        return ranked[0]["answer"]
