"""Omega reasoning helpers: structural causal model, goal inference, verification margins,
proof-carrying answers, a small planner and the auxiliary stores the decoding add-ons use.

Reference files (src/omnicoder/reasoning/): omega_causal.py:1-133 (SCM, do-interventions,
abductive score, value of information, query template), omega_intent.py:1-211 (goal posterior
from an utterance: a speaker-utility listener, plan-recognition bias, preference-memory update),
constraints.py:13-90 / omega_verifier.py:1-72 (per-modality verification margins and their
weighted combination), omega_pca.py:1-59 (proof-carrying answer record), omega_planner.py:1-69
(budgeted planner), templates.py:1-42 (embedding template bank), nss.py:1-69 (symbolic state
DSL), kv_hints.py, graph_speculative.py:1-32 (branch choice), alg_core.py:1-48 (algorithm hints).

Differences, on purpose: the SCM evaluates mechanisms in a topological order of the declared
parents (the reference iterates to a fixed point) and supports counterfactuals with additive
exogenous noise (abduction: noise = observed - mechanism(parents)); the planner is a UCT tree
search rather than a best-first frontier.
"""
from __future__ import annotations

import json
import math
import re
from dataclasses import asdict, dataclass, field
from typing import Any, Callable


# ----------------------------------------------------------------------------
# structural causal model
# ----------------------------------------------------------------------------
@dataclass
class Variable:
    name: str
    value: Any = None
    parents: list = field(default_factory=list)


class SCM:
    """Variables with mechanisms v = f(parent values) (+ exogenous noise u_v, additive)."""

    def __init__(self):
        self.variables: dict[str, Variable] = {}
        self.mechanisms: dict[str, Callable[[dict], Any]] = {}
        self.noise: dict[str, float] = {}

    def add_variable(self, name: str, value: Any = None, parents: list | None = None) -> None:
        self.variables[name] = Variable(name, value, list(parents or []))

    def add_mechanism(self, target: str, func: Callable[[dict], Any], parents: list | None = None) -> None:
        if target not in self.variables:
            self.add_variable(target)
        if parents is not None:
            self.variables[target].parents = list(parents)
        self.mechanisms[target] = func

    def order(self) -> list[str]:
        """Topological order of the variables (parents first); raises on a cycle."""
        indeg = {v: 0 for v in self.variables}
        kids: dict[str, list] = {v: [] for v in self.variables}
        for v, var in self.variables.items():
            for p in var.parents:
                if p not in self.variables:
                    raise KeyError(f"unknown parent {p!r} of {v!r}")
                indeg[v] += 1
                kids[p].append(v)
        ready = [v for v, d in indeg.items() if d == 0]
        out = []
        while ready:
            v = ready.pop(0)
            out.append(v)
            for k in kids[v]:
                indeg[k] -= 1
                if indeg[k] == 0:
                    ready.append(k)
        if len(out) != len(self.variables):
            raise ValueError("the causal graph has a cycle")
        return out

    def _run(self, fixed: dict, noise: dict) -> dict:
        vals = {k: v.value for k, v in self.variables.items()}
        vals.update(fixed)
        for v in self.order():
            if v in fixed or v not in self.mechanisms:
                continue
            out = self.mechanisms[v](vals)
            if v in noise and isinstance(out, (int, float)):
                out = out + noise[v]
            vals[v] = out
        return vals

    def forward(self) -> dict:
        vals = self._run({}, self.noise)
        for k, v in vals.items():
            self.variables[k].value = v
        return vals

    def do(self, interventions: dict) -> dict:
        """Values after do(X = x) for the given variables (descendants recomputed)."""
        return self._run(dict(interventions), self.noise)

    def abduce(self, evidence: dict) -> dict:
        """Exogenous noise of the numeric mechanisms that reproduces the observed values."""
        noise = dict(self.noise)
        vals = {k: v.value for k, v in self.variables.items()}
        for v in self.order():
            if v in self.mechanisms:
                pred = self.mechanisms[v](vals)
                if v in evidence and isinstance(pred, (int, float)) and isinstance(evidence[v], (int, float)):
                    noise[v] = evidence[v] - pred
                vals[v] = evidence.get(v, pred + noise.get(v, 0.0) if isinstance(pred, (int, float)) else pred)
            elif v in evidence:
                vals[v] = evidence[v]
        return noise

    def counterfactual(self, evidence: dict, interventions: dict) -> dict:
        """Abduction (noise from the evidence), action (do), prediction."""
        noise = self.abduce(evidence)
        base = {k: evidence[k] for k in evidence if k not in self.mechanisms}
        base.update(interventions)
        return self._run(base, noise)


def abductive_score(scm: SCM, observations: dict, tol: float = 1e-6) -> float:
    """Fraction of the observations that the model's forward values reproduce (numbers within tol)."""
    if not observations:
        return 1.0
    vals = scm._run({}, scm.noise)
    hit = 0
    for k, v in observations.items():
        got = vals.get(k)
        if isinstance(v, (int, float)) and isinstance(got, (int, float)):
            hit += abs(got - v) <= tol
        else:
            hit += got == v
    return hit / len(observations)


def value_of_information(uncertainties: dict, budget: int = 1, costs: dict | None = None) -> list[tuple]:
    """The `budget` variables with the largest uncertainty per unit cost."""
    costs = costs or {}
    items = sorted(uncertainties.items(), key=lambda kv: -kv[1] / max(1e-9, costs.get(kv[0], 1.0)))
    return items[:max(1, budget)]


def build_minimal_scm_for_query(query: str) -> SCM:
    """Goal clarity G, evidence E, plan feasibility P -> answer quality A = 0.33 G + 0.33 E + 0.34 P,
    with the reference's keyword conditioning of the query (why / how / cause -> G, code /
    compile / test -> P, cite / evidence / source -> E)."""
    scm = SCM()
    q = (query or "").lower()
    scm.add_variable("G", 0.7 if any(w in q for w in ("why", "how", "cause")) else 0.5)
    scm.add_variable("E", 0.7 if any(w in q for w in ("cite", "evidence", "source")) else 0.5)
    scm.add_variable("P", 0.7 if any(w in q for w in ("code", "compile", "test")) else 0.5)
    scm.add_mechanism("A", lambda v: min(1.0, max(0.0, 0.33 * v["G"] + 0.33 * v["E"] + 0.34 * v["P"])),
                      parents=["G", "E", "P"])
    return scm


# ----------------------------------------------------------------------------
# goal inference
# ----------------------------------------------------------------------------
GOALS = {
    "write_code": ("code", "function", "implement", "write", "program", "script", "class"),
    "explain": ("why", "how", "explain", "what", "describe"),
    "debug": ("bug", "error", "fix", "fails", "traceback", "crash"),
    "summarize": ("summarize", "summary", "tl;dr", "shorten", "brief"),
    "compute": ("calculate", "compute", "sum", "solve", "how many", "+", "*"),
    "prove": ("prove", "proof", "verify", "show that"),
    "translate": ("translate", "in french", "in spanish", "into"),
}


@dataclass
class GoalHypothesis:
    goal: str
    prior: float
    posterior: float


@dataclass
class GoalBelief:
    hypotheses: list = field(default_factory=list)
    constraints: list = field(default_factory=list)
    desiderata: list = field(default_factory=list)

    def top(self) -> str | None:
        return self.hypotheses[0].goal if self.hypotheses else None


def _softmax(xs: list[float]) -> list[float]:
    m = max(xs)
    e = [math.exp(x - m) for x in xs]
    s = sum(e)
    return [x / s for x in e]


def infer_goals(utterance: str, context: str | None = None, k: int = 3, alpha: float = 2.0,
                memory: dict | None = None) -> GoalBelief:
    """Posterior over latent goals: a listener that inverts a speaker who picks words that signal
    the goal (keyword utility, softmax with rationality alpha), times a plan-recognition term
    (longer, multi-step requests favour goals that need plans), times preference memory (past goal
    frequencies, as a Dirichlet-style prior update)."""
    u = (utterance or "").lower() + " " + (context or "").lower()
    goals = list(GOALS)
    util = [sum(1.0 for w in GOALS[g] if w in u) for g in goals]
    like = _softmax([alpha * x for x in util])
    steps = len(re.findall(r"\b(then|and then|after|first|finally|next)\b", u))
    plan = _softmax([0.5 * steps * (g in ("write_code", "debug", "prove")) for g in goals])
    mem = memory or {}
    tot = sum(mem.values())
    prior = [(1.0 + mem.get(g, 0.0)) / (len(goals) + tot) for g in goals]
    post = [a * b * c for a, b, c in zip(like, plan, prior)]
    s = sum(post)
    post = [p / s for p in post]
    order = sorted(range(len(goals)), key=lambda i: -post[i])[:max(1, k)]
    out = GoalBelief([GoalHypothesis(goals[i], prior[i], post[i]) for i in order])
    if "concise" in u or "brief" in u:
        out.desiderata.append("concise")
    if any(w in u for w in ("proof", "verify", "test")):
        out.constraints.append("must-verify")
    return out


# ----------------------------------------------------------------------------
# verification margins and proof-carrying answers
# ----------------------------------------------------------------------------
def _sig(z: float) -> float:
    return 1.0 / (1.0 + math.exp(-z))


def text_margin(hyp: str, context: str | None = None) -> float:
    """Token overlap of the hypothesis with its context over the smaller vocabulary (0.5 without one)."""
    if not hyp:
        return 0.0
    if not context:
        return 0.5
    h, c = set(hyp.lower().split()), set(context.lower().split())
    return min(1.0, len(h & c) / max(1, min(len(h), len(c))))


def code_margin(log: str | None = None, passed: int | None = None, total: int | None = None) -> float:
    if passed is not None and total:
        return max(0.0, min(1.0, passed / total))
    return 0.7 if log and ("ok" in log.lower() or "pass" in log.lower()) else 0.0


def unified_margin(signals: dict, weights: dict | None = None) -> float:
    """Weighted mean of per-modality margins; z-scored signals (image / video / audio) go through a
    sigmoid, margins in [0, 1] are used as they are."""
    w = weights or {}
    num = den = 0.0
    for name, v in signals.items():
        if v is None:
            continue
        m = _sig(v) if name.endswith("_z") else float(v)
        wt = w.get(name, 1.0)
        num += wt * m
        den += wt
    return num / den if den > 0 else 0.0


@dataclass
class Certificate:
    answer: str
    goal: dict
    signals: dict
    margin: float
    assumptions: list = field(default_factory=list)
    counterfactuals: list = field(default_factory=list)

    def to_json(self) -> str:
        return json.dumps(asdict(self), sort_keys=True, default=str)


def pack_certificate(answer: str, goal: GoalBelief | None, signals: dict | None, assumptions=None,
                     counterfactuals=None, weights: dict | None = None) -> Certificate:
    sig = dict(signals or {})
    g = {} if goal is None else {"top": goal.top(), "constraints": goal.constraints,
                                 "posterior": {h.goal: round(h.posterior, 4) for h in goal.hypotheses}}
    return Certificate(answer, g, sig, unified_margin(sig, weights), list(assumptions or []),
                       list(counterfactuals or []))


# ----------------------------------------------------------------------------
# planner, templates, symbolic state, KV hints, branch choice, algorithm hints
# ----------------------------------------------------------------------------
def plan_search(root, expand: Callable[[Any], list], step: Callable[[Any, Any], Any], value: Callable[[Any], float],
                budget: int = 64, max_depth: int = 4, c: float = 1.2):
    """UCT over actions: expand(state) -> actions, step(state, action) -> state, value(state) in
    [0, 1].  Returns (best first action, its mean value)."""
    stats: dict = {}                    # (path tuple) -> [visits, total]

    def rollout(state, path, depth):
        acts = expand(state) if depth < max_depth else []
        if not acts:
            v = value(state)
        else:
            n_parent = stats.get(path, [1, 0.0])[0]

            def ucb(a):
                n, t = stats.get(path + (a,), [0, 0.0])
                return float("inf") if n == 0 else t / n + c * math.sqrt(math.log(max(1, n_parent)) / n)
            a = max(acts, key=ucb)
            v = rollout(step(state, a), path + (a,), depth + 1)
        s = stats.setdefault(path, [0, 0.0])
        s[0] += 1
        s[1] += v
        return v

    for _ in range(max(1, budget)):
        rollout(root, (), 0)
    firsts = [(p[0], s) for p, s in stats.items() if len(p) == 1]
    if not firsts:
        return None, value(root)
    a, s = max(firsts, key=lambda kv: kv[1][0])
    return a, s[1] / s[0]


class TemplateBank:
    """Embedding -> payload store queried by cosine similarity."""

    def __init__(self):
        self.items: list[tuple[list, str]] = []

    def add(self, embedding, payload: str) -> None:
        self.items.append((list(map(float, embedding)), payload))

    def query(self, embedding, topk: int = 1, min_sim: float = 0.0) -> list[tuple[float, str]]:
        q = list(map(float, embedding))
        nq = math.sqrt(sum(x * x for x in q)) or 1.0
        out = []
        for e, p in self.items:
            ne = math.sqrt(sum(x * x for x in e)) or 1.0
            sim = sum(a * b for a, b in zip(q, e)) / (nq * ne)
            if sim >= min_sim:
                out.append((sim, p))
        return sorted(out, key=lambda t: -t[0])[:topk]


class SymbolicState:
    """Facts and goals edited by a line DSL (`fact: x`, `goal: y`, `retract: x`, `done: y`) and
    rendered as a context block for the prompt (the reference's NSS)."""

    def __init__(self):
        self.facts: list[str] = []
        self.goals: list[str] = []

    def apply(self, dsl: str) -> None:
        for line in dsl.splitlines():
            if ":" not in line:
                continue
            op, _, arg = line.partition(":")
            op, arg = op.strip().lower(), arg.strip()
            if op == "fact" and arg not in self.facts:
                self.facts.append(arg)
            elif op == "goal" and arg not in self.goals:
                self.goals.append(arg)
            elif op == "retract" and arg in self.facts:
                self.facts.remove(arg)
            elif op == "done" and arg in self.goals:
                self.goals.remove(arg)

    def render_context(self) -> str:
        return "\n".join([f"FACT {f}" for f in self.facts] + [f"GOAL {g}" for g in self.goals])


_KV_HINTS: dict = {}


def register_kv_hint(key: tuple, kv: Any, max_entries: int = 64) -> None:
    """Remember a prefix's KV state under its token tuple (oldest entry evicted past max_entries)."""
    if key in _KV_HINTS:
        _KV_HINTS.pop(key)
    _KV_HINTS[key] = kv
    while len(_KV_HINTS) > max_entries:
        _KV_HINTS.pop(next(iter(_KV_HINTS)))


def get_kv_hint(key: tuple):
    """The KV state of the longest registered prefix of `key` (None when there is none)."""
    for n in range(len(key), 0, -1):
        if key[:n] in _KV_HINTS:
            return key[:n], _KV_HINTS[key[:n]]
    return None


def select_branch(candidates: list[tuple[float, float, int]]) -> int:
    """candidates (log-prob, verifier score, branch id): the branch with the best sum of the two."""
    if not candidates:
        return -1
    return max(candidates, key=lambda c: c[0] + c[1])[2]


ALG_HINTS = {
    "sort": {"merge_sort": 0.6, "quick_sort": 0.4},
    "shortest path": {"dijkstra": 0.7, "bfs": 0.3},
    "graph": {"bfs": 0.5, "dfs": 0.5},
    "search": {"binary_search": 0.7, "linear_scan": 0.3},
    "substring": {"kmp": 0.5, "rolling_hash": 0.5},
    "subsequence": {"dynamic_programming": 1.0},
    "knapsack": {"dynamic_programming": 1.0},
    "schedule": {"greedy": 0.6, "heap": 0.4},
}


def algorithm_hints(prompt: str) -> dict:
    """Algorithm families the prompt's keywords point to, with weights (the reference's alg_core)."""
    p = (prompt or "").lower()
    return {k: v for k, v in ALG_HINTS.items() if k in p}
