"""Structured factor blending (SFB): prompt factorisation, belief propagation over goal
variables, a cache of compiled sum-product networks, fusion of factor messages into a
next-token bias, and a proof-margin arbiter -- the API the reference's generate() uses
(src/omnicoder/sfb/factorize.py:207-454, sfb/inference/bp.py, sfb/compile/spn.py:1-337,
sfb/fusion/cross_bias.py:1-168, sfb/arbiter.py:1-247), built here on
omnicoder.reasoning.factor_graph / omnicoder.reasoning.sfb without the reference's
optional AMR / SRL parsers (whose fallback is a pattern-based parse, as here).

  factorize_prompt(text) -> FactorizationResult(text, factors, goal_priors)
      factors: "subgoals" (numbered / bulleted / clause-split goals, each typed math /
      code / retrieval / text), "predicate_structure" (subject-relation-object triples from
      copula, possession and prepositional patterns), "entities" (quoted strings, numbers,
      capitalised words), "constraints" (must / should / never / at most N ...);
      goal_priors: per task family (code, math, sql, vqa, asr, retrieval) from keyword evidence.
  BeliefPropagation().run(result) -> messages: one binary variable per goal family with its
      prior as unary factor and pairwise factors coupling families that co-occur; the loopy-BP
      marginals weight each sub-goal's strings: [{"prefer_strings", "score", "goal"}].
  SPNCompiler: caches the compiled sum-product network (and the messages) per factor signature.
  CrossBiasFusion(encode_fn).bias(messages, vocab) -> [V] additive log-bias.
  ProofMarginArbiter: linear margin over verification evidence, accept / suggestions, decision
      log and logistic refit of its weights from that log.
"""
from __future__ import annotations

import json
import math
import re
from dataclasses import dataclass, field

import numpy as np
import torch

from ..reasoning.factor_graph import FactorGraph
from ..reasoning.sfb import SumProductNetwork, compile_factor_graph, cross_bias, factorize

GOAL_KEYWORDS = {
    "code": ("code", "python", "function", "compile", "unit test", "implement", "bug", "class "),
    "math": ("compute", "calculate", "sum", "integral", "solve", "equation", "prove", "number"),
    "sql": ("sql", "database", "query", "join", "table"),
    "vqa": ("image", "photo", "picture", "detect", "see in"),
    "asr": ("audio", "transcribe", "speech", "recording"),
    "retrieval": ("who", "when", "where", "cite", "source", "according"),
}
# goal families that tend to come together (pairwise coupling in the goal graph)
CO_OCCUR = (("code", "sql"), ("code", "math"), ("vqa", "retrieval"), ("asr", "retrieval"))


@dataclass
class Factor:
    name: str
    scope: tuple
    meta: dict = field(default_factory=dict)


@dataclass
class FactorizationResult:
    text: str
    factors: list
    goal_priors: dict


_TRIPLE = re.compile(r"\b([a-z][a-z0-9_]{1,24})\s+(is|are|has|have|of|for|to|in|on|with|from)\s+"
                     r"([a-z][a-z0-9_]{1,24})\b")
_CONSTRAINT = re.compile(r"\b(must|should|never|always|do not|don't|at most \d+|at least \d+|exactly \d+|"
                         r"no more than \d+)\b[^.;\n]*", re.I)


def goal_priors(text: str) -> dict:
    """Prior of each task family: 1 - 0.5 ** (keyword hits), so one hit gives 0.5, two 0.75."""
    low = text.lower()
    out = {}
    for g, kws in GOAL_KEYWORDS.items():
        hits = sum(low.count(k) for k in kws)
        if hits:
            out[g] = 1.0 - 0.5 ** hits
    return out


def factorize_prompt(text: str) -> FactorizationResult:
    factors = [Factor("subgoals", ("text",), {"goals": factorize(text)})]
    triples = [(m.group(1), m.group(2), m.group(3)) for m in _TRIPLE.finditer(text.lower())]
    if triples:
        factors.append(Factor("predicate_structure", ("text",), {"triples": triples}))
    ents = re.findall(r"\"([^\"]{1,64})\"|'([^']{1,64})'", text)
    ents = [a or b for a, b in ents] + re.findall(r"\b\d+(?:\.\d+)?\b", text) + \
        [w for w in re.findall(r"\b[A-Z][a-zA-Z0-9]{2,}\b", text)]
    if ents:
        factors.append(Factor("entities", ("text",), {"entities": list(dict.fromkeys(ents))}))
    cons = [m.group(0).strip() for m in _CONSTRAINT.finditer(text)]
    if cons:
        factors.append(Factor("constraints", ("text",), {"constraints": cons}))
    return FactorizationResult(text, factors, goal_priors(text))


def _signature(res: FactorizationResult) -> str:
    return json.dumps([(f.name, sorted(map(str, f.meta.items()))) for f in res.factors], sort_keys=True)


class SPNCompiler:
    """Compiled sum-product networks of goal graphs, cached by factor signature."""

    def __init__(self, capacity: int = 64):
        self.capacity = capacity
        self._spn: dict = {}
        self._msgs: dict = {}

    def maybe_compile(self, res: FactorizationResult) -> SumProductNetwork:
        key = _signature(res)
        if key not in self._spn:
            if len(self._spn) >= self.capacity:
                self._spn.clear()
                self._msgs.clear()
            names, factors = _goal_factors(res)
            self._spn[key] = compile_factor_graph({n: [0, 1] for n in names},
                                                  [(vs, (lambda t: (lambda *x: float(t[x])))(tab))
                                                   for vs, tab in factors])
        return self._spn[key]

    def lookup(self, res: FactorizationResult):
        return self._msgs.get(_signature(res))

    def register(self, res: FactorizationResult, messages: list) -> None:
        self._msgs[_signature(res)] = messages


def _goal_factors(res: FactorizationResult):
    """Binary goal variables (families with a prior) with unary and co-occurrence factors."""
    pri = res.goal_priors or {"text": 0.5}
    names = sorted(pri)
    factors = [((n,), np.array([1.0 - pri[n], pri[n]])) for n in names]
    pair = [(a, b) for a, b in CO_OCCUR if a in pri and b in pri]
    for a, b in pair:
        factors.append(((a, b), np.array([[1.0, 0.8], [0.8, 1.5]])))
    return names, factors


class BeliefPropagation:
    """Loopy sum-product over the goal graph; marginals weight the sub-goals' strings."""

    def __init__(self, iters: int = 30, damping: float = 0.2):
        self.iters, self.damping = iters, damping

    def marginals(self, res: FactorizationResult) -> dict:
        names, factors = _goal_factors(res)
        fg = FactorGraph()
        for n in names:
            fg.add_variable(n, 2)
        for vs, tab in factors:
            fg.add_factor(vs, tab)
        return {n: float(m[1]) for n, m in fg.marginals(self.iters, self.damping).items()}

    def run(self, res: FactorizationResult) -> list:
        marg = self.marginals(res)
        goals = next((f.meta["goals"] for f in res.factors if f.name == "subgoals"), [])
        fam = {"math": "math", "code": "code", "retrieval": "retrieval"}
        out = []
        for g in goals:
            w = marg.get(fam.get(g["kind"], ""), 0.5)
            out.append({"prefer_strings": [g["goal"]], "score": w, "goal": g["kind"]})
        for f in res.factors:
            if f.name == "entities":
                out.append({"prefer_strings": f.meta["entities"], "score": 0.5, "goal": "entities"})
        return out


class CrossBiasFusion:
    """Messages -> additive next-token log-bias: every message's strings become a token
    distribution (smoothed), mixed with the message scores as weights."""

    def __init__(self, encode_fn=None, floor: float = 1e-3, strength: float = 1.0):
        self.encode_fn, self.floor, self.strength = encode_fn, floor, strength

    def bias(self, messages: list, vocab: int, device=None) -> torch.Tensor | None:
        if self.encode_fn is None:
            raise RuntimeError("CrossBiasFusion needs encode_fn")
        probs, weights = [], []
        for m in messages:
            ids = [int(i) for s in m["prefer_strings"] for i in self.encode_fn(s) if 0 <= int(i) < vocab]
            if not ids or m["score"] <= 0:
                continue
            p = torch.full((vocab,), self.floor / vocab)
            p.index_add_(0, torch.tensor(ids), torch.full((len(ids),), (1.0 - self.floor) / len(ids)))
            probs.append(p)
            weights.append(float(m["score"]))
        if not probs:
            return None
        b = cross_bias(probs, weights, strength=self.strength)
        return b if device is None else b.to(device)


@dataclass
class ProofMarginInputs:
    llm_confidence: float
    sum_log_factors: float
    verifier_score: float
    retrieval_hits: int = 0
    code_passk: float = 0.0
    clip_z: float = 0.0
    audio_z: float = 0.0
    video_z: float = 0.0


_FIELDS = ("text", "code", "img", "audio", "video")


@dataclass
class ProofMarginArbiter:
    """margin = w_text (confidence + verifier) + sum log factors + w_code pass@k + w_img clip_z
    + w_audio audio_z + w_video video_z; an answer is accepted when margin >= threshold (0 when
    unset).  Low margins come with suggestions for the decoder."""
    w_text: float = 1.0
    w_code: float = 1.0
    w_img: float = 1.0
    w_audio: float = 1.0
    w_video: float = 1.0
    threshold: float | None = None
    log_path: str | None = None

    def compute_margin(self, x: ProofMarginInputs) -> float:
        return (self.w_text * (x.llm_confidence + x.verifier_score) + x.sum_log_factors + self.w_code * x.code_passk
                + self.w_img * x.clip_z + self.w_audio * x.audio_z + self.w_video * x.video_z)

    def accept(self, x: ProofMarginInputs) -> bool:
        return self.compute_margin(x) >= (self.threshold if self.threshold is not None else 0.0)

    def suggestions(self, x: ProofMarginInputs) -> dict:
        m = self.compute_margin(x)
        thr = self.threshold if self.threshold is not None else 0.0
        if m >= thr:
            return {}
        gap = thr - m
        out = {"escalate_block_verify": True, "disable_early_exit": True}
        if gap > 1.0:
            out["bump_scmoe_topk"] = True
        if x.retrieval_hits == 0:
            out["request_retrieval"] = True
        if x.verifier_score < 0.5:
            out["request_resolve"] = True
        return out

    def log_decision(self, x: ProofMarginInputs, accepted: bool) -> None:
        if self.log_path:
            with open(self.log_path, "a") as f:
                f.write(json.dumps({**x.__dict__, "accepted": bool(accepted)}) + "\n")

    @staticmethod
    def fit_weights_from_log(log_path: str, steps: int = 500, lr: float = 0.1) -> dict:
        """Logistic regression of the logged accept labels on (confidence + verifier, pass@k,
        clip_z, audio_z, video_z) with sum_log_factors as an offset; returns the five weights."""
        rows = [json.loads(l) for l in open(log_path) if l.strip()]
        if not rows:
            return {f"w_{k}": 1.0 for k in _FIELDS}
        X = np.array([[r["llm_confidence"] + r["verifier_score"], r["code_passk"], r["clip_z"], r["audio_z"],
                       r["video_z"]] for r in rows])
        off = np.array([r["sum_log_factors"] for r in rows])
        y = np.array([1.0 if r["accepted"] else 0.0 for r in rows])
        w = np.ones(X.shape[1])
        for _ in range(steps):
            p = 1.0 / (1.0 + np.exp(-(X @ w + off)))
            w -= lr * X.T @ (p - y) / len(rows)
        return {f"w_{k}": float(v) for k, v in zip(_FIELDS, w)}


def sfb_bias(text: str, encode_fn, vocab: int, device=None, spn: SPNCompiler | None = None,
             bp: BeliefPropagation | None = None, strength: float = 1.0) -> torch.Tensor | None:
    """The whole pipeline: factorise, (cached) belief propagation, fusion into a [V] bias."""
    res = factorize_prompt(text)
    spn = spn or SPNCompiler()
    msgs = spn.lookup(res)
    if msgs is None:
        spn.maybe_compile(res)
        msgs = (bp or BeliefPropagation()).run(res)
        spn.register(res, msgs)
    return CrossBiasFusion(encode_fn, strength=strength).bias(msgs, vocab, device)


__all__ = ["Factor", "FactorizationResult", "factorize_prompt", "goal_priors", "BeliefPropagation", "SPNCompiler",
           "CrossBiasFusion", "ProofMarginInputs", "ProofMarginArbiter", "sfb_bias"]
