"""Adaptive graph of thoughts, Omega controller, reflection, latent BFS and
answer certificates (reference src/omnicoder/reasoning/adaptive_graph.py:1-476,
omega_controller.py:1-135, reflection / latent search / certificates).

AdaptiveGraphOfThoughts: nodes are partial solutions; each round expands the
best `beam` frontier nodes with `propose(state) -> [states]`, merges duplicates
(by `key(state)`) keeping the best score, and stops when `is_final` holds or the
budget runs out; scores come from `score(state) -> float`.
OmegaController: maps the uncertainty of the next-token distribution
(normalised entropy) to decoding knobs -- temperature, top-k, whether to
invoke search -- with hysteresis.
reflect: generate -> critique -> revise loop until the critic accepts.
latent_bfs: breadth-first search over a latent transition function with a
goal predicate.
verify_certificate: checks an answer certificate (numeric equality within a
tolerance, or a python assertion run in the sandbox).
"""
from __future__ import annotations

import math
from collections import deque
from dataclasses import dataclass, field
from typing import Callable


@dataclass
class ThoughtNode:
    state: object
    score: float
    depth: int
    parents: list = field(default_factory=list)


class AdaptiveGraphOfThoughts:
    def __init__(self, propose: Callable, score: Callable, is_final: Callable, key: Callable = repr,
                 beam: int = 3, max_rounds: int = 8, max_nodes: int = 200):
        self.propose, self.score, self.is_final, self.key = propose, score, is_final, key
        self.beam, self.max_rounds, self.max_nodes = beam, max_rounds, max_nodes
        self.nodes: dict = {}

    def run(self, root):
        r = ThoughtNode(root, self.score(root), 0)
        self.nodes = {self.key(root): r}
        frontier = [r]
        best = r
        for _ in range(self.max_rounds):
            new = []
            for n in sorted(frontier, key=lambda x: -x.score)[:self.beam]:
                for s in self.propose(n.state):
                    k = self.key(s)
                    sc = self.score(s)
                    if k in self.nodes:                       # merge: keep the best score, add a parent
                        m = self.nodes[k]
                        m.parents.append(n)
                        m.score = max(m.score, sc)
                        continue
                    child = ThoughtNode(s, sc, n.depth + 1, [n])
                    self.nodes[k] = child
                    new.append(child)
                    if self.is_final(s) and (not self.is_final(best.state) or sc > best.score):
                        best = child
                    if len(self.nodes) >= self.max_nodes:
                        return best
            if not new or self.is_final(best.state):
                break
            frontier = new
            top = max(new, key=lambda x: x.score)
            if not self.is_final(best.state) and top.score > best.score:
                best = top
        return best


class OmegaController:
    def __init__(self, low: float = 0.3, high: float = 0.7, base_temperature: float = 0.7):
        self.low, self.high, self.t0 = low, high, base_temperature
        self.mode = "normal"

    @staticmethod
    def normalized_entropy(probs) -> float:
        import torch
        p = probs.float().clamp_min(1e-12)
        return float(-(p * p.log()).sum(-1).mean() / math.log(p.shape[-1]))

    def knobs(self, probs) -> dict:
        h = self.normalized_entropy(probs)
        if self.mode == "normal" and h > self.high:
            self.mode = "explore"
        elif self.mode == "explore" and h < self.low:
            self.mode = "normal"
        if self.mode == "explore":
            return {"temperature": self.t0 * 1.3, "top_k": 64, "search": True, "entropy": h}
        return {"temperature": self.t0 * (0.5 + h), "top_k": 20, "search": False, "entropy": h}


def reflect(generate: Callable[[str], str], critique: Callable[[str, str], tuple], prompt: str,
            max_rounds: int = 3) -> tuple[str, int]:
    """critique(prompt, answer) -> (accepted: bool, feedback: str); the feedback is appended to the prompt."""
    ans = generate(prompt)
    for r in range(max_rounds):
        ok, fb = critique(prompt, ans)
        if ok:
            return ans, r
        ans = generate(f"{prompt}\n# feedback: {fb}\n")
    return ans, max_rounds


def latent_bfs(start, step: Callable, goal: Callable, key: Callable = repr, max_states: int = 10000):
    """step(state) -> [(action, next_state)]; returns the action path to the first goal state (or None)."""
    q = deque([(start, [])])
    seen = {key(start)}
    while q and len(seen) <= max_states:
        s, path = q.popleft()
        if goal(s):
            return path
        for a, n in step(s):
            k = key(n)
            if k not in seen:
                seen.add(k)
                q.append((n, path + [a]))
    return None


def verify_certificate(answer, certificate: dict) -> bool:
    kind = certificate.get("kind")
    if kind == "numeric":
        from ..training.rl import reward_numeric
        return reward_numeric(str(answer), certificate["value"], certificate.get("tol", 1e-6)) == 1.0
    if kind == "python":
        from ..training.rl import run_sandboxed
        rc, _ = run_sandboxed(f"answer = {answer!r}\n{certificate['check']}\n")
        return rc == 0
    raise ValueError(f"unknown certificate kind {kind!r}")
